// NUQ codebook fitting on the GPU: the Fisher-weighted 1-D k-means of
// train_nuq_codebook (kvquant/quant/nuq.py:6-44), part of the kvq_lib.cu unity build.
//
// The reference runs scikit-learn KMeans (k-means++ seeding, n_init=10, max_iter=100)
// on the host. In one dimension the optimal clusters are intervals of the sorted
// samples, so this path solves the problem directly instead of by local search:
//   1. range:    per-CTA min / max of the samples;
//   2. hist:     one HBM pass puts every sample into one of kCbBins equal bins over
//                [min, max]; per bin the sum of weights and the sum of weight times
//                offset from the bin centre (shared-memory histogram per CTA, one
//                partial histogram per CTA, no global atomics);
//   3. reduce:   bin sums over the CTAs in double;
//   4. solve:    the best split of the sorted bins into K contiguous clusters:
//                maximise sum_k S_k^2 / W_k (S = weighted sum, W = weight; the
//                within-cluster sum of squares is sum w x^2 minus that), dynamic
//                programming over clusters, each layer filled with the monotone
//                split-point rule (divide and conquer, valid because the 1-D sum of
//                squares obeys the quadrangle inequality); one CTA, prefix sums in
//                shared memory;
//   5. refine:   exact Lloyd steps on the raw samples from that optimum (nearest
//                centre, then weighted mean), which also split the bins that hold a
//                cluster boundary. A Lloyd step never raises the sum of squares.
// The result is the bin-level global optimum refined on the samples; k-means++ with
// restarts can only match it up to the width of a bin.
#pragma once
#include "kvq_common.cuh"

namespace kvq {

constexpr int kCbBins = 8192;          // histogram bins over [min, max]
constexpr int kCbMaxK = 16;            // 4-bit codebooks
constexpr int kCbMaxGrid = 148;        // one histogram CTA per SM at most
constexpr int64_t kCbPerCta = 65536;   // samples per histogram CTA before the grid grows
constexpr int kCbHistThreads = 1024;
constexpr int kCbRefineThreads = 256;
constexpr int kCbSolveThreads = 1024;
constexpr int kCbMaxRefine = 64;
constexpr int kCbStreamMul = 4;        // range / refine CTAs per histogram CTA

inline int cb_grid(int64_t n) {
  int64_t g = (n + kCbPerCta - 1) / kCbPerCta;
  return (int)(g < 1 ? 1 : (g > kCbMaxGrid ? kCbMaxGrid : g));
}

// Bin geometry, computed in fp32 once (histogram block 0) and read by the later kernels.
struct CbBins {
  float lo, h, inv_h;
};

struct CbLayout {
  size_t mm, bins, hist, wsum, ssum, drow, arg, cen, ref, total;
};

inline CbLayout cb_layout(int64_t n) {
  const int G = cb_grid(n);
  CbLayout L{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o += (bytes + 255) & ~size_t(255);
    return at;
  };
  L.mm = take(sizeof(float2) * kCbStreamMul * G);
  L.bins = take(sizeof(CbBins));
  L.hist = take(sizeof(double) * 2 * kCbBins * (size_t)G);
  L.wsum = take(sizeof(double) * kCbBins);
  L.ssum = take(sizeof(double) * kCbBins);
  L.drow = take(sizeof(double) * (kCbBins + 1));
  L.arg = take(sizeof(int) * (kCbMaxK + 1) * (size_t)(kCbBins + 1));
  L.cen = take(sizeof(double) * kCbMaxK);
  L.ref = take(sizeof(double) * 2 * kCbMaxK * (size_t)(kCbStreamMul * G));
  L.total = o;
  return L;
}

// Min / max over the range kernel's per-CTA partials (whole block; exact, so every
// CTA that calls it gets the same bins), then the bin geometry.
__device__ inline CbBins cb_bins_block(const float2* mm, int Gm) {
  __shared__ float rlo[32], rhi[32];
  float lo = INFINITY, hi = -INFINITY;
  for (int g = threadIdx.x; g < Gm; g += blockDim.x) {
    lo = fminf(lo, mm[g].x);
    hi = fmaxf(hi, mm[g].y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const int warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  if ((threadIdx.x & 31) == 0) {
    rlo[warp] = lo;
    rhi[warp] = hi;
  }
  __syncthreads();
  lo = rlo[0];
  hi = rhi[0];
  for (int i = 1; i < nw; ++i) {
    lo = fminf(lo, rlo[i]);
    hi = fmaxf(hi, rhi[i]);
  }
  CbBins b{lo, 0.f, 0.f};
  const float span = __fsub_rn(hi, lo);
  if (span > 0.f) {
    b.h = __fdiv_rn(span, (float)kCbBins);
    b.inv_h = __fdiv_rn((float)kCbBins, span);
    if (!(b.inv_h < INFINITY)) b.h = b.inv_h = 0.f;  // span below the fp32 range: one bin
  }
  return b;
}

__device__ __forceinline__ int cb_bin(const CbBins& b, float v) {
  int k = (int)__fmul_rn(__fsub_rn(v, b.lo), b.inv_h);
  return k < 0 ? 0 : (k >= kCbBins ? kCbBins - 1 : k);
}

__device__ __forceinline__ float cb_centre(const CbBins& b, int k) {
  return __fadd_rn(b.lo, __fmul_rn((float)k + 0.5f, b.h));
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Visits every sample once over the grid: 16-byte loads of x and w when both are
// 16-byte aligned (two per thread in flight), scalar loads for the rest.
template <class F>
__device__ __forceinline__ void cb_for_each(const float* __restrict__ x,
                                            const float* __restrict__ w, int64_t n, F&& f) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t start = 0;
  if ((((uintptr_t)x | (uintptr_t)w) & 15) == 0) {
    const int64_t n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    for (int64_t i = gid; i < n4; i += 2 * stride) {
      const float4 a0 = x4[i], b0 = w4[i];
      const bool two = i + stride < n4;
      float4 a1 = a0, b1 = b0;
      if (two) {
        a1 = x4[i + stride];
        b1 = w4[i + stride];
      }
      f(a0.x, b0.x); f(a0.y, b0.y); f(a0.z, b0.z); f(a0.w, b0.w);
      if (two) {
        f(a1.x, b1.x); f(a1.y, b1.y); f(a1.z, b1.z); f(a1.w, b1.w);
      }
    }
    start = n4 << 2;
  }
  for (int64_t i = start + gid; i < n; i += stride) f(x[i], w[i]);
}

// Bits of status[0] (status words cleared by the host before the range kernel).
enum CbStatus : int { kCbFewBins = 1, kCbBadSample = 2, kCbBadWeight = 4 };

// 1. Per-CTA min / max; flags a NaN or infinite sample.
__global__ void __launch_bounds__(256) cb_range_kernel(const float* __restrict__ x, int64_t n,
                                                       float2* __restrict__ mm,
                                                       int32_t* __restrict__ status) {
  float lo = INFINITY, hi = -INFINITY;
  bool bad = false;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t start = 0;
  if (((uintptr_t)x & 15) == 0) {
    const int64_t n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int64_t i = gid; i < n4; i += stride) {
      const float4 a = x4[i];
      lo = fminf(fminf(lo, a.x), fminf(a.y, fminf(a.z, a.w)));
      hi = fmaxf(fmaxf(hi, a.x), fmaxf(a.y, fmaxf(a.z, a.w)));
      bad |= !(isfinite(a.x) && isfinite(a.y) && isfinite(a.z) && isfinite(a.w));
    }
    start = n4 << 2;
  }
  for (int64_t i = start + gid; i < n; i += stride) {
    const float v = x[i];
    lo = fminf(lo, v);
    hi = fmaxf(hi, v);
    bad |= !isfinite(v);
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(&status[0], kCbBadSample);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  __shared__ float slo[8], shi[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    slo[warp] = lo;
    shi[warp] = hi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < 8; ++i) {
      lo = fminf(lo, slo[i]);
      hi = fmaxf(hi, shi[i]);
    }
    mm[blockIdx.x] = make_float2(lo, hi);
  }
}

// 2. Per-CTA weighted histogram: part[cta][0][bin] = sum w, part[cta][1][bin] = sum w*(x - centre),
// accumulated in double (a CTA adds up to n / 148 samples into a bin; fp32 sums of that
// length lose 1e-4 .. 1e-3 relative in concentrated bins).
__global__ void __launch_bounds__(kCbHistThreads) cb_hist_kernel(const float* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 int64_t n,
                                                                 const float2* __restrict__ mm,
                                                                 int Gm, CbBins* __restrict__ bins_out,
                                                                 double* __restrict__ part,
                                                                 int32_t* __restrict__ status) {
  extern __shared__ double cb_hist_sh[];  // [2][kCbBins]
  double* sw = cb_hist_sh;
  double* sd = cb_hist_sh + kCbBins;
  for (int i = threadIdx.x; i < 2 * kCbBins; i += blockDim.x) cb_hist_sh[i] = 0.0;
  const CbBins bins = cb_bins_block(mm, Gm);  // ends with a block barrier
  if (blockIdx.x == 0 && threadIdx.x == 0) *bins_out = bins;
  bool bad = false;
  cb_for_each(x, w, n, [&](float v, float wt) {
    const int k = cb_bin(bins, v);
    bad |= !(wt >= 0.f && wt < INFINITY);
    atomicAdd(&sw[k], (double)wt);
    atomicAdd(&sd[k], (double)wt * (double)__fsub_rn(v, cb_centre(bins, k)));
  });
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(&status[0], kCbBadWeight);
  double* out = part + (size_t)blockIdx.x * 2 * kCbBins;
  for (int i = threadIdx.x; i < 2 * kCbBins; i += blockDim.x) out[i] = cb_hist_sh[i];
}

// 3. Bin sums over the CTAs (double, fixed order); status[1] counts the occupied bins.
__global__ void __launch_bounds__(256) cb_reduce_kernel(const double* __restrict__ part, int G,
                                                        const CbBins* __restrict__ bins_in,
                                                        double* __restrict__ wsum,
                                                        double* __restrict__ ssum,
                                                        int32_t* __restrict__ status) {
  const CbBins bins = *bins_in;
  const int k = blockIdx.x * blockDim.x + threadIdx.x;  // grid covers kCbBins exactly
  double W = 0.0, D = 0.0;
#pragma unroll 8
  for (int g = 0; g < G; ++g) {
    const double* p = part + (size_t)g * 2 * kCbBins;
    W += p[k];
    D += p[kCbBins + k];
  }
  wsum[k] = W;
  ssum[k] = D + (double)cb_centre(bins, k) * W;
  const int occ = __syncthreads_count(W > 0.0);
  if (threadIdx.x == 0 && occ) atomicAdd(&status[1], occ);
}

__device__ __forceinline__ double cb_gain(const double* PW, const double* PS, int i, int j) {
  const double wt = PW[j] - PW[i];
  const double s = PS[j] - PS[i];
  return wt > 0.0 ? s * s / wt : 0.0;
}

// 4. Optimal K-interval split of the bins (one CTA). drow: one DP row of
// kCbBins+1 doubles; arg[l][j]: best start of the l-th cluster for bins [0, j).
constexpr size_t kCbSolveSmem =
    sizeof(double) * 3 * (kCbBins + 1) + ((sizeof(unsigned short) * (kCbBins + 1) + 7) & ~7ul);
__global__ void __launch_bounds__(kCbSolveThreads, 1)
    cb_solve_kernel(const double* __restrict__ wsum, const double* __restrict__ ssum, int K,
                    const CbBins* __restrict__ bins_in, double* __restrict__ drow,
                    int* __restrict__ arg, double* __restrict__ centres, float* __restrict__ out,
                    int32_t* __restrict__ status) {
  constexpr int NB = kCbBins;
  constexpr int per = NB / kCbSolveThreads;
  extern __shared__ double cb_solve_sh[];
  double* PW = cb_solve_sh;                 // [NB + 1] prefix weight
  double* PS = cb_solve_sh + (NB + 1);      // [NB + 1] prefix weighted sum
  double* PV = cb_solve_sh + 2 * (NB + 1);  // [NB + 1] previous DP layer
  unsigned short* A16 = reinterpret_cast<unsigned short*>(cb_solve_sh + 3 * (NB + 1));
  __shared__ double wtot[32], stot[32], slot_v[32];
  __shared__ int slot_i[32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int flags = status[0];
  if (flags || status[1] < K) {  // bad input, or fewer occupied bins than clusters
    if (t == 0 && !flags) status[0] = kCbFewBins;
    return;
  }
  // Exclusive block scan of the per-thread totals of `per` consecutive bins.
  double tw = 0.0, ts = 0.0;
  for (int i = 0; i < per; ++i) {
    tw += wsum[t * per + i];
    ts += ssum[t * per + i];
  }
  double iw = tw, is = ts;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double a = __shfl_up_sync(0xffffffffu, iw, o);
    const double b = __shfl_up_sync(0xffffffffu, is, o);
    if (lane >= o) {
      iw += a;
      is += b;
    }
  }
  if (lane == 31) {
    wtot[warp] = iw;
    stot[warp] = is;
  }
  __syncthreads();
  if (warp == 0) {
    double a = wtot[lane], b = stot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double a2 = __shfl_up_sync(0xffffffffu, a, o);
      const double b2 = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) {
        a += a2;
        b += b2;
      }
    }
    wtot[lane] = a;
    stot[lane] = b;
  }
  __syncthreads();
  double bw = (warp ? wtot[warp - 1] : 0.0) + iw - tw;
  double bs = (warp ? stot[warp - 1] : 0.0) + is - ts;
  if (t == 0) {
    PW[0] = 0.0;
    PS[0] = 0.0;
  }
  for (int i = 0; i < per; ++i) {
    bw += wsum[t * per + i];
    bs += ssum[t * per + i];
    PW[t * per + i + 1] = bw;
    PS[t * per + i + 1] = bs;
  }
  __syncthreads();

  // Layer 1: one cluster over bins [0, j).
  for (int j = t; j <= NB; j += kCbSolveThreads) PV[j] = cb_gain(PW, PS, 0, j);
  __syncthreads();

  // Layer l: D_l[j] = max_{i <= j} D_{l-1}[i] + gain(i, j), best i monotone in j.
  // j = NB first, then the midpoints j = s(2m+1) for s = NB/2 .. 1, whose split
  // points lie between those of j - s and j + s (already filled). Every level uses
  // the whole block: a group of L threads per midpoint (L = 1024 / midpoints, at
  // least 1), the group's threads striding its candidate range. D_{l-1} (PV) and the
  // layer's split points (A16) are in shared memory; D_l goes to `drow`.
  for (int l = 2; l <= K; ++l) {
    int* A = arg + (size_t)l * (NB + 1);
    if (t == 0) {
      drow[0] = 0.0;
      A[0] = 0;
      A16[0] = 0;
    }
    for (int s = NB; s >= 1; s >>= 1) {
      const int count = (s == NB) ? 1 : NB / (2 * s);
      const int L = count >= kCbSolveThreads ? 1 : kCbSolveThreads / count;
      for (int base = 0; base < count * L; base += kCbSolveThreads) {
        const int g = base + t;
        const int m = g / L, r = g - m * L;
        const int j = (s == NB) ? NB : s * (2 * m + 1);
        int lo = 0, hi = j;
        if (s != NB) {
          lo = (m == 0) ? 0 : (int)A16[j - s];
          hi = min((int)A16[j + s], j);
          if (hi < lo) hi = lo;  // rounding broke monotonicity: scan the lower bound only
        }
        double best = -1.0;
        int bi = lo;
#pragma unroll 4
        for (int i = lo + r; i <= hi; i += L) {
          const double v = PV[i] + cb_gain(PW, PS, i, j);
          if (v > best) {
            best = v;
            bi = i;
          }
        }
        for (int o = (L < 32 ? L : 32) >> 1; o > 0; o >>= 1) {  // within the group's lanes
          const double ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ob > best || (ob == best && oi < bi)) {
            best = ob;
            bi = oi;
          }
        }
        if (L > 32) {  // count < 32: a single pass, so the barrier is uniform
          if (lane == 0) {
            slot_v[warp] = best;
            slot_i[warp] = bi;
          }
          __syncthreads();
          if (warp == 0) {  // lane q holds warp q's result; midpoint lane / nw owns nw lanes
            const int nw = L >> 5;
            double bb = slot_v[lane];
            int ii = slot_i[lane];
            for (int o = nw >> 1; o > 0; o >>= 1) {
              const double ob = __shfl_xor_sync(0xffffffffu, bb, o);
              const int oi = __shfl_xor_sync(0xffffffffu, ii, o);
              if (ob > bb || (ob == bb && oi < ii)) {
                bb = ob;
                ii = oi;
              }
            }
            if ((lane & (nw - 1)) == 0) {
              const int mm = lane / nw;
              const int jj = (s == NB) ? NB : s * (2 * mm + 1);
              drow[jj] = bb;
              A[jj] = ii;
              A16[jj] = (unsigned short)ii;
            }
          }
        } else if (r == 0) {
          drow[j] = best;
          A[j] = bi;
          A16[j] = (unsigned short)bi;
        }
      }
      __syncthreads();
    }
    if (l < K) {
      for (int j = t; j <= NB; j += kCbSolveThreads) PV[j] = drow[j];
      __syncthreads();
    }
  }

  // Backtrack the K intervals; their weighted means are the centres (ascending).
  if (t == 0) {
    const CbBins bins = *bins_in;
    int j = NB;
    for (int l = K; l >= 1; --l) {
      const int i = (l == 1) ? 0 : arg[(size_t)l * (NB + 1) + j];
      const double wt = PW[j] - PW[i];
      double c = wt > 0.0 ? (PS[j] - PS[i]) / wt
                          : (double)bins.lo + 0.5 * (double)(i + j) * (double)bins.h;
      centres[l - 1] = c;
      out[l - 1] = (float)c;
      j = i;
    }
  }
}

// 5a. One Lloyd step on the samples: per-CTA sums of w and w*(x - c_k) per nearest centre.
template <int K>
__global__ void __launch_bounds__(kCbRefineThreads) cb_refine_kernel(
    const float* __restrict__ x, const float* __restrict__ w, int64_t n,
    const double* __restrict__ centres, double* __restrict__ part,
    const int32_t* __restrict__ status) {
  if (status[0]) return;
  __shared__ float acc[2 * K][kCbRefineThreads];  // per-thread slots: no sharing, no atomics
  __shared__ float cs[K];
  const int t = threadIdx.x;
  if (t < K) cs[t] = (float)centres[t];
#pragma unroll
  for (int k = 0; k < 2 * K; ++k) acc[k][t] = 0.f;
  __syncthreads();
  float mid[K > 1 ? K - 1 : 1];
#pragma unroll
  for (int k = 0; k + 1 < K; ++k) mid[k] = 0.5f * (cs[k] + cs[k + 1]);
  cb_for_each(x, w, n, [&](float v, float wt) {
    int j = 0;
#pragma unroll
    for (int k = 0; k + 1 < K; ++k) j += (v > mid[k]) ? 1 : 0;
    acc[j][t] += wt;
    acc[K + j][t] += wt * (v - cs[j]);
  });
  __syncthreads();
  const int warp = t >> 5, lane = t & 31;
  for (int s = warp; s < 2 * K; s += kCbRefineThreads / 32) {
    double v = 0.0;
    for (int i = lane; i < kCbRefineThreads; i += 32) v += (double)acc[s][i];
    v = warp_sum_d(v);
    if (lane == 0) part[(size_t)blockIdx.x * 2 * K + s] = v;
  }
}

// 5b. New centres = old + sum w*(x - c) / sum w (an empty cluster keeps its centre).
// One warp per cluster (lanes stride the CTAs' partials), kCbMaxK warps.
__global__ void __launch_bounds__(32 * kCbMaxK) cb_finalize_kernel(
    const double* __restrict__ part, int G, int K, double* __restrict__ centres,
    float* __restrict__ out, const int32_t* __restrict__ status) {
  if (status[0]) return;
  __shared__ double cn[kCbMaxK];
  const int k = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (k < K) {
    double W = 0.0, D = 0.0;
    for (int g = lane; g < G; g += 32) {
      W += part[(size_t)g * 2 * K + k];
      D += part[(size_t)g * 2 * K + K + k];
    }
    W = warp_sum_d(W);
    D = warp_sum_d(D);
    if (lane == 0) {
      const double c = (double)(float)centres[k];
      cn[k] = W > 0.0 ? c + D / W : centres[k];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // a Lloyd step keeps 1-D centres in order; sort anyway for the output
    for (int a = 1; a < K; ++a) {
      const double v = cn[a];
      int b = a - 1;
      while (b >= 0 && cn[b] > v) {
        cn[b + 1] = cn[b];
        --b;
      }
      cn[b + 1] = v;
    }
    for (int a = 0; a < K; ++a) {
      centres[a] = cn[a];
      out[a] = (float)cn[a];
    }
  }
}

template <int K>
int launch_refine(const float* x, const float* w, int64_t n, int Gm, const CbLayout& L,
                  char* ws, float* out, int32_t* status, int iters, cudaStream_t s) {
  double* cen = reinterpret_cast<double*>(ws + L.cen);
  double* ref = reinterpret_cast<double*>(ws + L.ref);
  for (int r = 0; r < iters; ++r) {
    cb_refine_kernel<K><<<Gm, kCbRefineThreads, 0, s>>>(x, w, n, cen, ref, status);
    cb_finalize_kernel<<<1, 32 * kCbMaxK, 0, s>>>(ref, Gm, K, cen, out, status);
  }
  return check_launch("fit_codebook(refine)");
}

}  // namespace kvq

extern "C" size_t kvq_fit_codebook_workspace(int64_t n) {
  return kvq::cb_layout(n < 1 ? 1 : n).total;
}

extern "C" int kvq_fit_codebook(const float* x, const float* weights, int64_t n, int bits,
                                int refine_iters, float* centres, void* workspace,
                                size_t workspace_bytes, int32_t* status, void* stream) {
  using namespace kvq;
  clear_error();
  if (!x || !weights || !centres || !status || n < 1) {
    set_error("fit_codebook: null pointer or n=%lld < 1", (long long)n);
    return KVQ_ERR_INVALID;
  }
  if (bits < 1 || bits > 4) {
    set_error("fit_codebook: bits=%d outside 1..4", bits);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (refine_iters < 0 || refine_iters > kCbMaxRefine) {
    set_error("fit_codebook: refine_iters=%d outside 0..%d", refine_iters, kCbMaxRefine);
    return KVQ_ERR_INVALID;
  }
  const CbLayout L = cb_layout(n);
  if (!workspace || workspace_bytes < L.total || ((uintptr_t)workspace & 255)) {
    set_error("fit_codebook: workspace needs %zu bytes, 256-byte aligned", L.total);
    return KVQ_ERR_INVALID;
  }
  const int K = 1 << bits;
  const int G = cb_grid(n);
  const int Gm = kCbStreamMul * G;
  cudaStream_t s = as_stream(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  float2* mm = reinterpret_cast<float2*>(ws + L.mm);
  double* hist = reinterpret_cast<double*>(ws + L.hist);
  double* wsum = reinterpret_cast<double*>(ws + L.wsum);
  double* ssum = reinterpret_cast<double*>(ws + L.ssum);
  CbBins* bins = reinterpret_cast<CbBins*>(ws + L.bins);
  const size_t hist_smem = sizeof(double) * 2 * kCbBins;
  const size_t solve_smem = kCbSolveSmem;
  cudaFuncSetAttribute(cb_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)hist_smem);
  cudaFuncSetAttribute(cb_solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)solve_smem);
  if (cudaMemsetAsync(status, 0, 2 * sizeof(int32_t), s) != cudaSuccess) {
    set_error("fit_codebook: clearing status: %s", cudaGetErrorString(cudaGetLastError()));
    return KVQ_ERR_CUDA;
  }
  cb_range_kernel<<<Gm, 256, 0, s>>>(x, n, mm, status);
  cb_hist_kernel<<<G, kCbHistThreads, hist_smem, s>>>(x, weights, n, mm, Gm, bins, hist, status);
  cb_reduce_kernel<<<kCbBins / 256, 256, 0, s>>>(hist, G, bins, wsum, ssum, status);
  cb_solve_kernel<<<1, kCbSolveThreads, solve_smem, s>>>(
      wsum, ssum, K, bins, reinterpret_cast<double*>(ws + L.drow),
      reinterpret_cast<int*>(ws + L.arg), reinterpret_cast<double*>(ws + L.cen), centres,
      status);
  int rc = check_launch("fit_codebook");
  if (rc || refine_iters == 0) return rc;
  switch (K) {
    case 2: return launch_refine<2>(x, weights, n, Gm, L, ws, centres, status, refine_iters, s);
    case 4: return launch_refine<4>(x, weights, n, Gm, L, ws, centres, status, refine_iters, s);
    case 8: return launch_refine<8>(x, weights, n, Gm, L, ws, centres, status, refine_iters, s);
    default: return launch_refine<16>(x, weights, n, Gm, L, ws, centres, status, refine_iters, s);
  }
}
