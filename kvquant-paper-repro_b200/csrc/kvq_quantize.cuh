// Quantize-on-append for a prefill block: KVQuantizer.quantize_k / quantize_v
// (kvquant/quant/kv_quantizer.py:72-122) with dense-and-sparse outliers
// (kvquant/quant/dense_sparse.py:4-32), writing the packed cache layout.
//
// Keys are quantized per channel: outliers are the top-k |n| along tokens of
// each (batch, channel) column, k = max(1, int((S - sink) * ratio)). Values are
// quantized per token: scale/zero and the top-k run over all C channels of the
// token row. Top-k selection is an exact radix select on the fp32 bits of |n|;
// among values equal to the k-th largest, lower token (keys) / channel
// (values) indices are taken first.
#pragma once
#include "kvq_common.cuh"

namespace kvq {

// Per-column / per-row selection result.
struct Select {
  uint32_t thr;     // fp32 bits of the k-th largest |n|
  int32_t kleft;    // remaining rank inside the current radix prefix
  int32_t tie_cut;  // |n| == thr is selected iff index <= tie_cut
  int32_t ties;     // number of entries equal to thr (last radix pass)
};

__device__ __forceinline__ uint32_t abs_bits(float n) { return __float_as_uint(n) & 0x7fffffffu; }

__device__ __forceinline__ bool selected(uint32_t ab, int32_t idx, const Select& s) {
  return ab > s.thr || (ab == s.thr && idx <= s.tie_cut);
}

// ---------------------------------------------------------------------------
// Decisions in input space. For one (zero, scale) pair (a key channel or a
// value token) n(x) = fl(fl(x - zero) / fl(scale + 1e-8)) is non-decreasing in
// x, so for fp16 inputs every decision the emit step takes on n -- outlier
// (|n| > thr, or |n| == thr subject to the tie cut), and the dense code
// si[#(tau <= clamp(n))] -- is a comparison of x's order against a few fp16
// boundaries found once by bisection over the fp16 order with the exact n.
// ord16 maps fp16 bits to a monotone integer (both zeros to 0); finite inputs
// lie in [-31743, 31743]. Non-finite inputs take the per-element path.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ord16(uint32_t h) {
  return (h & 0x8000u) ? -(int)(h & 0x7fffu) : (int)(h & 0x7fffu);
}
__device__ __forceinline__ float ord16_value(int o) {
  const unsigned short hb = o < 0 ? (unsigned short)(0x8000 | -o) : (unsigned short)o;
  return __half2float(__ushort_as_half(hb));
}

// Outlier boundaries (int4 {op, om, tpa, tmb}): |n| > thr <=> o >= op || o <= om,
// |n| == thr <=> o in [tpa, op) or (om, tmb]; so out(x) <=> o >= op || o <= om ||
// ((o >= tpa || o <= tmb) && index <= cut). op = kNoOrder marks a (zero, scale)
// pair where the decisions do not apply (non-positive or non-finite divisor).
constexpr int kNoOrder = -1000000;

// Smallest finite order o in [lo, hi] with pred(n(o)) true (pred monotone
// false -> true), or hi + 1 if none.
template <class P>
__device__ __forceinline__ int first_order(int lo, int hi, const Normalizer& nz, P pred) {
  int a = lo, b = hi + 1;  // pred false below a, true from b
  while (a < b) {
    const int m = a + ((b - a) >> 1);
    if (pred(nz(ord16_value(m)))) b = m; else a = m + 1;
  }
  return a;
}

// Whether input-space decisions apply to (zero, scale): the divisor must be
// positive and finite (then n is monotone in x).
__device__ __forceinline__ bool xspace_ok(float zero, float scale) {
  const float b = __fadd_rn(scale, 1e-8f);
  return b > 0.f && b < INFINITY && fabsf(zero) < INFINITY;
}

// One of the four outlier boundaries (which = 0..3: op, om, tpa, tmb).
__device__ inline int out_bound(const Normalizer& nz, uint32_t thr_bits, int which) {
  constexpr int kLo = -31743, kHi = 31743;
  const float thr = __uint_as_float(thr_bits);
  switch (which) {
    case 0: return first_order(kLo, kHi, nz, [&](float n) { return n > thr; });
    case 1: return first_order(kLo, kHi, nz, [&](float n) { return n >= -thr; }) - 1;
    case 2: return first_order(kLo, kHi, nz, [&](float n) { return n >= thr; });
    default: return first_order(kLo, kHi, nz, [&](float n) { return n > -thr; }) - 1;
  }
}

__device__ __forceinline__ bool out_by_order(int o, const int4& ob, int32_t idx, int32_t cut) {
  return o >= ob.x || o <= ob.y || ((o >= ob.z || o <= ob.w) && idx <= cut);
}

// ---------------------------------------------------------------------------
// Keys: radix select along tokens, per (b, channel) column.
// Columns are numbered col = b * CL + c, CL = n_heads * 128 local channels.
// ---------------------------------------------------------------------------
struct KeyShape {
  const __half* k;
  int64_t B, S, C_full, c0, CL;  // c0 = first local channel in the full row
  int64_t off;                   // 1 when token 0 is the sink, else 0
  const float* scale;            // [C_full]
  const float* zero;
};


constexpr int kHistCols = 32;  // columns per histogram CTA

constexpr int kHistUnroll = 8;  // rows in flight per thread

// Histogram of the radix digit at `shift` of |n| among entries matching the
// prefix so far. grid = (CL/32 column groups, B, row blocks); block 256: lane =
// column (a warp reads 64 contiguous bytes of a row), warp w takes rows w,
// w + 8, ... with 8 loads in flight. Rows of the shared histogram are padded
// to 257 words so that lanes adding the same digit hit distinct banks.
__global__ void __launch_bounds__(256) key_hist_kernel(KeyShape ks, int shift,
                                                       const Select* __restrict__ sel,
                                                       uint32_t* __restrict__ hist,
                                                       int64_t rows_per_block) {
  __shared__ uint32_t h[kHistCols][257];
  for (int i = threadIdx.x; i < kHistCols * 257; i += blockDim.x) (&h[0][0])[i] = 0;
  __syncthreads();
  const int64_t b = blockIdx.y;
  const int64_t cg = (int64_t)blockIdx.x * kHistCols;
  const int lc = threadIdx.x & 31;  // column inside the group
  const int warp = threadIdx.x >> 5;
  const int64_t c = cg + lc;
  const int64_t col = b * ks.CL + c;
  const uint32_t mask_hi = shift >= 24 ? 0u : (0xffffffffu << (shift + 8));
  const uint32_t prefix = sel[col].thr & mask_hi;
  Normalizer nz;
  nz.init(ks.zero[ks.c0 + c], ks.scale[ks.c0 + c]);
  const int64_t n_rest = ks.S - ks.off;
  const int64_t r0 = (int64_t)blockIdx.z * rows_per_block;
  const int64_t r1 = min(n_rest, r0 + rows_per_block);
  const __half* xcol = ks.k + (b * ks.S + ks.off) * ks.C_full + ks.c0 + c;
  for (int64_t rb = r0 + warp; rb < r1; rb += 8 * kHistUnroll) {
    __half xv[kHistUnroll];
#pragma unroll
    for (int i = 0; i < kHistUnroll; ++i) {
      const int64_t r = rb + 8 * i;
      xv[i] = r < r1 ? xcol[r * ks.C_full] : __float2half(0.f);
    }
#pragma unroll
    for (int i = 0; i < kHistUnroll; ++i) {
      if (rb + 8 * i < r1) {
        const uint32_t ab = abs_bits(nz(__half2float(xv[i])));
        if ((ab & mask_hi) == prefix) atomicAdd(&h[lc][(ab >> shift) & 0xffu], 1u);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kHistCols * 256; i += blockDim.x) {
    const uint32_t v = h[i >> 8][i & 255];
    if (v) atomicAdd(&hist[(b * ks.CL + cg + (i >> 8)) * 256 + (i & 255)], v);
  }
}

// One thread per column: picks the digit holding the k-th largest entry.
__global__ void key_select_kernel(Select* __restrict__ sel, uint32_t* __restrict__ hist,
                                  int64_t ncols, int shift) {
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= ncols) return;
  uint32_t* hc = hist + col * 256;
  Select s = sel[col];
  int32_t k = s.kleft;
  int d = 255;
  for (; d > 0; --d) {
    const int32_t n = (int32_t)hc[d];
    if (k <= n) break;
    k -= n;
  }
  s.thr |= (uint32_t)d << shift;
  s.kleft = k;
  s.ties = (int32_t)hc[d];
  sel[col] = s;
  for (int i = 0; i < 256; ++i) hc[i] = 0;  // ready for the next pass
}

// Columns where only some of the entries equal to thr are taken (kleft <
// ties): the tie cut is the token index of the kleft-th entry equal to thr in
// token order; other columns take every tie (tie_cut = INT_MAX). Two kernels:
// key_ties_count_kernel counts each column's ties per row block (grid and load
// pattern of key_hist_kernel; CTAs whose 32 columns all take every tie skip),
// key_ties_find_kernel (one warp per column) finds the row block holding the
// cut from those counts and walks only that block's rows in order.
constexpr int kTieBlocksMax = 256;  // row blocks per column (the counts reuse the histogram)

inline int64_t tie_rows_per_block(int64_t n_rest) {
  const int64_t r = (n_rest + kTieBlocksMax - 1) / kTieBlocksMax;
  return r < 4096 ? 4096 : r;
}

__global__ void __launch_bounds__(256) key_ties_count_kernel(KeyShape ks,
                                                             const Select* __restrict__ sel,
                                                             int32_t* __restrict__ counts,
                                                             int64_t rows_per_block, int nrb) {
  __shared__ int32_t s_cnt[8][32];
  const int64_t b = blockIdx.y;
  const int64_t cg = (int64_t)blockIdx.x * kHistCols;
  const int lc = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = cg + lc;
  const int64_t col = b * ks.CL + c;
  const Select s0 = sel[col];
  if (!__syncthreads_or(s0.kleft < s0.ties)) return;
  Normalizer nz;
  nz.init(ks.zero[ks.c0 + c], ks.scale[ks.c0 + c]);
  const int64_t n_rest = ks.S - ks.off;
  const int64_t r0 = (int64_t)blockIdx.z * rows_per_block;
  const int64_t r1 = min(n_rest, r0 + rows_per_block);
  const __half* xcol = ks.k + (b * ks.S + ks.off) * ks.C_full + ks.c0 + c;
  int cnt = 0;
  for (int64_t rb = r0 + warp; rb < r1; rb += 8 * kHistUnroll) {
    __half xv[kHistUnroll];
#pragma unroll
    for (int i = 0; i < kHistUnroll; ++i) {
      const int64_t r = rb + 8 * i;
      xv[i] = r < r1 ? xcol[r * ks.C_full] : __float2half(0.f);
    }
#pragma unroll
    for (int i = 0; i < kHistUnroll; ++i)
      if (rb + 8 * i < r1 && abs_bits(nz(__half2float(xv[i]))) == s0.thr) ++cnt;
  }
  s_cnt[warp][lc] = cnt;
  __syncthreads();
  if (warp == 0) {
    int t = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += s_cnt[w][lc];
    counts[col * nrb + blockIdx.z] = t;
  }
}

__global__ void __launch_bounds__(256) key_ties_find_kernel(KeyShape ks, Select* __restrict__ sel,
                                                            const int32_t* __restrict__ counts,
                                                            int64_t rows_per_block, int nrb,
                                                            int64_t ncols) {
  const int64_t col = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (col >= ncols) return;
  Select s = sel[col];
  if (s.kleft >= s.ties) {
    if (lane == 0) { s.tie_cut = 0x7fffffff; sel[col] = s; }
    return;
  }
  // the row block where the running tie count reaches kleft
  int32_t need = s.kleft;
  int rb = -1;
  for (int i0 = 0; i0 < nrb && rb < 0; i0 += 32) {
    const int i = i0 + lane;
    const int32_t v = i < nrb ? counts[col * nrb + i] : 0;
    int32_t incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    const uint32_t hit = __ballot_sync(0xffffffffu, incl >= need);
    if (hit) {
      const int L = __ffs(hit) - 1;
      need -= __shfl_sync(0xffffffffu, incl - v, L);
      rb = i0 + L;
    } else {
      need -= __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  int32_t cut = -1;
  if (rb >= 0) {
    const int64_t b = col / ks.CL, c = col % ks.CL;
    Normalizer nz;
    nz.init(ks.zero[ks.c0 + c], ks.scale[ks.c0 + c]);
    const int64_t n_rest = ks.S - ks.off;
    const int64_t r0 = (int64_t)rb * rows_per_block;
    const int64_t r1 = min(n_rest, r0 + rows_per_block);
    const __half* xcol = ks.k + (b * ks.S + ks.off) * ks.C_full + ks.c0 + c;
    for (int64_t q0 = r0; q0 < r1 && need > 0; q0 += 32) {
      const int64_t r = q0 + lane;
      const bool tie =
          r < r1 && abs_bits(nz(__half2float(xcol[r * ks.C_full]))) == s.thr;
      const uint32_t bal = __ballot_sync(0xffffffffu, tie);
      const int n = __popc(bal);
      if (n >= need) {
        uint32_t m = bal;
        for (int k = 1; k < need; ++k) m &= m - 1;
        cut = (int32_t)(q0 + __ffs(m) - 1);
        need = 0;
      } else {
        need -= n;
      }
    }
  }
  if (lane == 0) { s.tie_cut = cut; sel[col] = s; }
}

// ---------------------------------------------------------------------------
// Values: one CTA per (b, token) row, thread i holding channels 16i..16i+15 in
// registers: per-token min/max over all C_full channels, then the exact top-k
// of |n| over those channels.
// ---------------------------------------------------------------------------
constexpr int kValRowMax = 16384;  // channels per value row
constexpr int kPlanEPT = 16;       // channels per thread

// Radix-select step shared by the plan kernels (warp 0): the digit holding the
// kleft-th largest entry. Walking the bins from 255 down, the first d >= 1
// whose suffix count reaches kleft (d = 0 if none). Lane L holds bins
// 8L..8L+7; a suffix scan over the lanes finds the one lane where the count
// crosses kleft, which then walks its own 8 bins.
__device__ __forceinline__ void radix_pick(const uint32_t* hist, int32_t* sh_kleft,
                                           int32_t* sh_digit, int32_t* sh_ties) {
  const int L = threadIdx.x & 31;
  const int32_t k0 = *sh_kleft;
  int32_t h8[8], s8 = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    h8[j] = (int32_t)hist[8 * L + j];
    s8 += h8[j];
  }
  int32_t suf = s8;  // bins 8L .. 255
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t v = __shfl_down_sync(0xffffffffu, suf, o);
    if (L + o < 32) suf += v;
  }
  const int32_t above = suf - s8;  // bins 8L+8 .. 255
  const bool mine = (k0 <= suf && (L == 31 || above < k0)) || (L == 0 && k0 > suf);
  if (mine) {
    int32_t k = k0 - above;
    int d = 0;  // bin 0 is the fall-through: it is never tested
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      if (8 * L + j == 0) break;
      if (k <= h8[j]) { d = 8 * L + j; break; }
      k -= h8[j];
    }
    *sh_kleft = k;
    *sh_digit = d;
    *sh_ties = (int32_t)hist[d];
  }
}

// Radix select of the kleft-th largest among n words u[0..n) that share
// `prefix` (which has no bits below shift0 + 8), digits at shift0, shift0 - 8, ... 0; every
// thread of the CTA takes part. Returns the threshold; sh_kleft / sh_ties end
// as the remaining rank among the entries equal to it and their count.
__device__ uint32_t radix_select_list(const uint32_t* u, int n, uint32_t prefix, int shift0,
                                      uint32_t* hist, int32_t* sh_kleft, int32_t* sh_digit,
                                      int32_t* sh_ties) {
  for (int shift = shift0; shift >= 0; shift -= 8) {
    const uint32_t mask_hi = shift >= 24 ? 0u : (0xffffffffu << (shift + 8));
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t ab = u[i];
      if ((ab & mask_hi) == prefix) atomicAdd(&hist[(ab >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) radix_pick(hist, sh_kleft, sh_digit, sh_ties);
    __syncthreads();
    prefix |= (uint32_t)*sh_digit << shift;
    __syncthreads();
  }
  return prefix;
}

// The same select by one warp (no block barriers): for the short candidate
// lists of the value plan's fast path.
__device__ uint32_t radix_select_list_warp(const uint32_t* u, int n, uint32_t prefix, int shift0,
                                           uint32_t* hist, int32_t* sh_kleft, int32_t* sh_digit,
                                           int32_t* sh_ties) {
  const int lane = threadIdx.x & 31;
  for (int shift = shift0; shift >= 0; shift -= 8) {
    const uint32_t mask_hi = shift >= 24 ? 0u : (0xffffffffu << (shift + 8));
    for (int i = lane; i < 256; i += 32) hist[i] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const uint32_t ab = u[i];
      if ((ab & mask_hi) == prefix) atomicAdd(&hist[(ab >> shift) & 0xffu], 1u);
    }
    __syncwarp();
    radix_pick(hist, sh_kleft, sh_digit, sh_ties);
    __syncwarp();
    prefix |= (uint32_t)*sh_digit << shift;
    __syncwarp();
  }
  return prefix;
}

// Tie cut by one warp: the index (or chan[index]) of the need-th entry of
// list[0..n) equal to thr, INT_MAX when need is 0.
__device__ int32_t tie_cut_warp(const uint32_t* list, const uint32_t* chan, int n, uint32_t thr,
                                int32_t need) {
  const int lane = threadIdx.x & 31;
  int32_t cut = 0x7fffffff;
  for (int i0 = 0; i0 < n && need > 0; i0 += 32) {
    const int i = i0 + lane;
    const bool tie = i < n && list[i] == thr;
    const uint32_t bal = __ballot_sync(0xffffffffu, tie);
    const int cnt = __popc(bal);
    if (cnt >= need) {
      uint32_t m = bal;
      for (int k = 1; k < need; ++k) m &= m - 1;
      const int at = i0 + (__ffs(m) - 1);
      cut = chan ? (int32_t)chan[at] : at;
      need = 0;
    } else {
      need -= cnt;
    }
  }
  return cut;
}

// Block-wide reductions of the plan kernel (any blockDim multiple of 32).
// Max of a and of b over the block in one pass (two barriers).
__device__ __forceinline__ float2 plan_block_max2(float a, float b, float2* red) {
  a = warp_max(a);
  b = warp_max(b);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[w] = make_float2(a, b);
  __syncthreads();
  float2 r = make_float2(-INFINITY, -INFINITY);
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) {
    r.x = fmaxf(r.x, red[k].x);
    r.y = fmaxf(r.y, red[k].y);
  }
  __syncthreads();
  return r;
}

__device__ __forceinline__ float plan_block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = -INFINITY;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) r = fmaxf(r, red[k]);
  __syncthreads();
  return r;
}

// Fast path: the threshold lies in one of the 8 highest occupied binades
// (fp32 exponents) of |n|, found from per-thread counts; the entries of that
// binade are compacted in channel order and radix-selected on their low 24
// bits. Otherwise (or when the binade holds more than C_full / 2 entries) the
// whole row is radix-selected from shared memory.
__global__ void __launch_bounds__(1024) value_plan_kernel(
    const __half* __restrict__ v, int64_t B, int64_t S, int64_t C_full, int64_t off,
    int64_t kv, float* __restrict__ v_scale, float* __restrict__ v_zero, int64_t ld_stats,
    Select* __restrict__ sel, int32_t* __restrict__ counts, int64_t h0, int64_t n_heads,
    int64_t nt_cap) {
  extern __shared__ uint32_t vsm[];  // C_full words: the row's |n| bits, or a candidate list
  __shared__ uint32_t hist[256];
  __shared__ float red[32];
  __shared__ float2 red2[32];
  __shared__ int32_t s_bc[32][8];  // per-warp counts of the top binades
  __shared__ int32_t sh_kleft, sh_digit, sh_ties, sh_cut, sh_bin, sh_m;
  __shared__ uint32_t sh_thr;
  const int64_t row = blockIdx.x;  // over B * (S - off)
  const int64_t n_rest = S - off;
  const int64_t b = row / n_rest, t = row % n_rest + off;
  const __half* x = v + (b * S + t) * C_full;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int64_t c0 = (int64_t)kPlanEPT * tid;
  uint4 raw[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh)
    raw[hh] = c0 + 8 * hh < C_full ? *reinterpret_cast<const uint4*>(x + c0 + 8 * hh)
                                   : make_uint4(0u, 0u, 0u, 0u);
  const __half* xh = reinterpret_cast<const __half*>(raw);
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int e = 0; e < kPlanEPT; ++e) {
    if (c0 + e < C_full) {
      const float f = __half2float(xh[e]);
      mn = fminf(mn, f);
      mx = fmaxf(mx, f);
    }
  }
  {
    const float2 r = plan_block_max2(-mn, mx, reinterpret_cast<float2*>(red2));
    mn = -r.x;
    mx = r.y;
  }
  // kv_quantizer.py:106-107: scale = (max - min) / 2, zero = (max + min) / 2 (fp32).
  const float scale = __fdiv_rn(__fsub_rn(mx, mn), 2.0f);
  const float zero = __fdiv_rn(__fadd_rn(mx, mn), 2.0f);
  if (tid == 0) {
    v_scale[b * ld_stats + t] = scale;
    v_zero[b * ld_stats + t] = zero;
  }
  uint32_t u[kPlanEPT];
  int emax_t = -1;
  Normalizer nz;
  nz.init(zero, scale);
  const bool quick = nz.fast && finite8(raw[0]) && finite8(raw[1]);
#pragma unroll
  for (int e = 0; e < kPlanEPT; ++e) {
    const float xv = __half2float(xh[e]);
    const float n = quick ? nz.quot(xv) : __fdiv_rn(__fsub_rn(xv, nz.z), nz.b);
    u[e] = c0 + e < C_full ? abs_bits(n) : 0u;
    if (c0 + e < C_full) emax_t = max(emax_t, (int)(u[e] >> 23));
  }
  if (kv <= 0) {  // no outliers: a threshold nothing reaches
    if (tid == 0) {
      Select s;
      s.thr = 0xffffffffu;
      s.kleft = 0;
      s.ties = 0;
      s.tie_cut = 0x7fffffff;
      sel[b * S + t] = s;
    }
    return;
  }
  const int emax = (int)plan_block_max((float)emax_t, red);
  // counts of binades emax - j, j = 0..7 (8-bit fields; at most 16 per thread)
  uint64_t pk = 0ull;
#pragma unroll
  for (int e = 0; e < kPlanEPT; ++e) {
    const int j = emax - (int)(u[e] >> 23);
    if (c0 + e < C_full && j < 8) pk += 1ull << (8 * j);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int cj = __reduce_add_sync(0xffffffffu, (unsigned)((pk >> (8 * j)) & 0xffull));
    if (lane == 0) s_bc[w][j] = cj;
  }
  __syncthreads();
  const int cap = (int)(C_full / 2);
  if (tid == 0) {
    int cum = 0, bin = -1, m = 0;
    for (int j = 0; j < 8 && bin < 0; ++j) {
      int cj = 0;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) cj += s_bc[k][j];
      if (cum + cj >= kv) { bin = j; m = cj; } else { cum += cj; }
    }
    if (bin >= 0 && m > cap) bin = -1;
    sh_bin = bin;
    sh_m = m;
    sh_kleft = (int32_t)(bin >= 0 ? kv - cum : kv);  // the whole row from the top otherwise
  }
  __syncthreads();
  const int bin = sh_bin;
  uint32_t thr;
  const uint32_t* list;
  const uint32_t* chan = nullptr;  // channel of each list entry (fast path)
  int n;
  if (bin >= 0) {
    // compact the binade's entries in channel order: u at vsm[0..m), channel at vsm[cap..)
    const uint32_t eb = (uint32_t)(emax - bin);
    int mc = 0;
#pragma unroll
    for (int e = 0; e < kPlanEPT; ++e) mc += (c0 + e < C_full && (u[e] >> 23) == eb) ? 1 : 0;
    int incl = mc;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    if (lane == 31) s_bc[w][0] = incl;
    __syncthreads();
    int pos = incl - mc;
    for (int k = 0; k < w; ++k) pos += s_bc[k][0];
#pragma unroll
    for (int e = 0; e < kPlanEPT; ++e) {
      if (c0 + e < C_full && (u[e] >> 23) == eb) {
        vsm[pos] = u[e];
        vsm[cap + pos] = (uint32_t)(c0 + e);
        ++pos;
      }
    }
    __syncthreads();
    list = vsm;
    chan = vsm + cap;
    n = sh_m;
    // one warp selects among the binade's entries and finds the tie cut: bits
    // 31..24 are fixed by the binade; the first digit (bits 23..16) holds its
    // exponent's low bit, the same for every entry of the list
    if (tid < 32) {
      const uint32_t th =
          radix_select_list_warp(list, n, (eb >> 1) << 24, 16, hist, &sh_kleft, &sh_digit, &sh_ties);
      const int32_t cut = sh_kleft < sh_ties ? tie_cut_warp(list, chan, n, th, sh_kleft)
                                              : 0x7fffffff;
      if (lane == 0) {
        sh_thr = th;
        sh_cut = cut;
      }
    }
    __syncthreads();
    thr = sh_thr;
  } else {
#pragma unroll
    for (int e = 0; e < kPlanEPT; ++e)
      if (c0 + e < C_full) vsm[c0 + e] = u[e];
    __syncthreads();
    list = vsm;
    n = (int)C_full;
    thr = radix_select_list(list, n, 0u, 24, hist, &sh_kleft, &sh_digit, &sh_ties);
    // tie cut: the channel index of the kleft-th entry equal to the threshold
    if (tid < 32) {
      const int32_t cut = sh_kleft < sh_ties ? tie_cut_warp(list, nullptr, n, thr, sh_kleft)
                                              : 0x7fffffff;
      if (lane == 0) sh_cut = cut;
    }
    __syncthreads();
  }
  if (tid == 0) {
    Select s;
    s.thr = thr;
    s.kleft = sh_kleft;
    s.ties = sh_ties;
    s.tie_cut = sh_cut;
    sel[b * S + t] = s;
  }
  // Outlier counts of the token's heads in [h0, h0 + n_heads), added into the
  // CSR row of (unit, tile, 16-token block) (counts[row + 1], zeroed by the
  // caller): the 8 threads of a head (16 channels each) sum their selections.
  if (counts) {
    const int32_t cut = sh_cut;
    int cnt = 0;
#pragma unroll
    for (int e = 0; e < kPlanEPT; ++e)
      cnt += (c0 + e < C_full && (u[e] > thr || (u[e] == thr && (int32_t)(c0 + e) <= cut))) ? 1 : 0;
    cnt += __shfl_xor_sync(0xffffffffu, cnt, 1);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, 2);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, 4);
    const int64_t hf = c0 / kHeadDim;
    if ((tid & 7) == 0 && cnt > 0 && c0 < C_full && hf >= h0 && hf < h0 + n_heads) {
      const int64_t unit = b * n_heads + (hf - h0);
      atomicAdd(counts + 2 * (unit * nt_cap + t / kTileTokens) + (t % kTileTokens) / 16 + 1, cnt);
    }
  }
}

// One packed outlier entry: position (token_in_tile << 7 | channel) in the low
// 16 bits; in the high 16 bits the reference's dequantized value at that
// position, fp16((cb[c0] + n) * s + z) (kv_quantizer.py:89,117; c0 = the code
// of a dense 0, n the normalized outlier), which the decode kernels use in
// place of the dequantized dense code there. An outlier key or value then
// enters the attention exactly as the reference's fp16 K_hat / V_hat holds it
// (for an unclamped input this is the input itself), where a rounded n would
// be off by up to 2^-12 |n| s.
__device__ __forceinline__ uint32_t outlier_entry(int token, int channel, float value) {
  const __half h = __float2half_rn(value);
  return (uint32_t)((token << 7) | channel) | ((uint32_t)__half_as_ushort(h) << 16);
}

// Nearest centroid of a clamped dense value v in [-1, 1] by exact switching
// points. Sorted centroids sv[0..n-1] (original indices si); when every gap
// between neighbours exceeds two ulps of (1 + max |c|), two distances
// fl(|v - c|) to different centroids on the same side of v never round to the
// same value, so the first-minimum rule of kvquant_ops.cu:141-148 picks one of
// the two neighbours of v, and which one is monotone in v. tau[k] is then the
// smallest fp32 v for which sorted position k + 1 wins over k (found by
// bisection over the fp32 order), and the code is si[#(tau <= v)].
struct NearestTable {
  float tau[16];
  uint8_t si[16];
  int fast;  // 0: a gap is too small, use nearest_centroid_sorted
};

// Orders fp32 values as integers (monotone for all non-NaN floats).
__device__ __forceinline__ int32_t f2ord(float f) {
  const int32_t i = __float_as_int(f);
  return i >= 0 ? i : (int32_t)(0x80000000u - (uint32_t)i);
}
__device__ __forceinline__ float ord2f(int32_t o) {
  return __int_as_float(o >= 0 ? o : (int32_t)(0x80000000u - (uint32_t)o));
}

// Built by one warp from the sorted codebook (lane k bisects tau[k]).
__device__ void build_nearest_table(const float* sv, const uint8_t* si, int n, NearestTable* t) {
  const int k = threadIdx.x & 31;
  float m = fmaxf(fabsf(sv[0]), fabsf(sv[n - 1])) + 1.f;
  int ex;
  frexpf(m, &ex);  // m < 2^ex: distances below m have ulp <= 2^(ex - 24)
  const float ulp2 = ldexpf(1.f, ex - 23);
  bool ok = true;
  if (k < n - 1) ok = __fsub_rn(sv[k + 1], sv[k]) > ulp2;
  const bool fast = __all_sync(0xffffffffu, ok);
  if (k < n - 1 && fast) {
    // predicate(v): position k + 1 chosen over k; false at sv[k], true at sv[k + 1]
    const float lo_c = sv[k], hi_c = sv[k + 1];
    const bool hi_first = si[k + 1] < si[k];  // wins ties
    int64_t lo = f2ord(lo_c), hi = f2ord(hi_c);
    while (hi - lo > 1) {
      const int64_t mid = lo + (hi - lo) / 2;
      const float v = ord2f((int32_t)mid);
      const float dl = fabsf(__fsub_rn(v, lo_c)), dh = fabsf(__fsub_rn(v, hi_c));
      const bool up = dh < dl || (dh == dl && hi_first);
      if (up) hi = mid; else lo = mid;
    }
    t->tau[k] = ord2f((int32_t)hi);
  }
  if (k < n) t->si[k] = si[k];
  if (k == 0) t->fast = fast ? 1 : 0;
}

// Sorted position of an input's code: #(cbnd[k] <= o) over the code bounds.
template <int BITS>
__device__ __forceinline__ int pos_by_order(int o, const int16_t* cbnd, int stride = 1) {
  int pos = 0;
#pragma unroll
  for (int step = 1 << (BITS - 1); step >= 1; step >>= 1)
    if (cbnd[(pos + step - 1) * stride] <= o) pos += step;
  return pos;
}

// The codebook as the emit and bound kernels use it, prepared once per call:
// original and sorted values, the sorted entries' original indices, the
// switching points and the code of a dense 0.
struct __align__(16) EmitCodebook {
  float cb[16], cbs[16];
  uint8_t cbi[16];
  NearestTable nt;
  int c0;
  int pad[6];
};
static_assert(sizeof(EmitCodebook) % 16 == 0, "copied as 16-byte words");

__global__ void codebook_setup_kernel(const float* __restrict__ cb, int bits,
                                      EmitCodebook* __restrict__ out) {
  __shared__ EmitCodebook e;
  const int ncb = 1 << bits;
  if (threadIdx.x == 0) {
    for (int k = 0; k < 16; ++k) e.cb[k] = k < ncb ? cb[k] : 0.f;
    sort_codebook(e.cb, ncb, e.cbs, e.cbi);
    e.c0 = nearest_centroid(0.f, e.cb, ncb);
  }
  __syncwarp();
  build_nearest_table(e.cbs, e.cbi, ncb, &e.nt);
  __syncwarp();
  for (int i = threadIdx.x; i < (int)(sizeof(EmitCodebook) / 4); i += 32)
    reinterpret_cast<uint32_t*>(out)[i] = reinterpret_cast<const uint32_t*>(&e)[i];
}

// Copies an EmitCodebook from global to shared memory (all threads, then sync).
__device__ __forceinline__ void load_emit_codebook(const EmitCodebook* g, EmitCodebook* s) {
  for (int i = threadIdx.x; i < (int)(sizeof(EmitCodebook) / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(s)[i] = reinterpret_cast<const uint4*>(g)[i];
  __syncthreads();
}

// Outlier bounds of every value token (thread = (token, bound)); tokens before
// `off` (the sink) have none.
__global__ void value_out_bounds_kernel(const float* __restrict__ v_zero,
                                        const float* __restrict__ v_scale, int64_t ld,
                                        const Select* __restrict__ sel, int64_t B, int64_t S,
                                        int64_t off, int4* __restrict__ obnd) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * S * 4) return;
  const int64_t row = i >> 2, b = row / S, t = row % S;
  if (t < off) return;
  const float z = v_zero[b * ld + t], sc = v_scale[b * ld + t];
  int v = kNoOrder;
  if (xspace_ok(z, sc)) {
    Normalizer nz;
    nz.init(z, sc);
    v = out_bound(nz, sel[row].thr, (int)(i & 3));
  }
  reinterpret_cast<int*>(obnd)[i] = v;
}

// Outlier bounds of every key column [B * CL] (thread = (column, bound)).
__global__ void key_out_bounds_kernel(KeyShape ks, const Select* __restrict__ sel,
                                      int4* __restrict__ obnd, int64_t ncols) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ncols * 4) return;
  const int64_t col = i >> 2, c = col % ks.CL;
  const float z = ks.zero[ks.c0 + c], sc = ks.scale[ks.c0 + c];
  int v = kNoOrder;
  if (xspace_ok(z, sc)) {
    Normalizer nz;
    nz.init(z, sc);
    v = out_bound(nz, sel[col].thr, (int)(i & 3));
  }
  reinterpret_cast<int*>(obnd)[i] = v;
}

// Code bounds of n_groups (zero, scale) pairs: group g uses zero/scale at
// (g / per_row) * ld + g % per_row (keys: the CL channels, per_row = CL;
// values: the tokens (b, t), per_row = S, ld = the stats' row stride).
// cbnd[g][k] (k < 2^bits - 1) = the smallest fp16 order whose dense value
// reaches tau[k]; cbnd[g][15] = 1 where the bounds are valid.
__global__ void __launch_bounds__(256) code_bounds_kernel(const float* __restrict__ zero,
                                                          const float* __restrict__ scale,
                                                          int64_t n_groups, int64_t per_row,
                                                          int64_t ld,
                                                          const EmitCodebook* __restrict__ ecb,
                                                          int bits, int16_t* __restrict__ cbnd) {
  __shared__ EmitCodebook s_ec;
  load_emit_codebook(ecb, &s_ec);
  const NearestTable& s_nt = s_ec.nt;
  const int ncb = 1 << bits;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_groups * 16) return;
  const int64_t g = i >> 4;
  const int k = (int)(i & 15);
  const int64_t zi = (g / per_row) * ld + g % per_row;
  const float z = zero[zi], sc = scale[zi];
  const bool ok = s_nt.fast != 0 && xspace_ok(z, sc);
  int16_t v = 0;
  if (k == 15) {
    v = ok ? 1 : 0;
  } else if (ok && k < ncb - 1) {
    Normalizer nz;
    nz.init(z, sc);
    const float tau = s_nt.tau[k];
    v = (int16_t)first_order(-31743, 31743, nz,
                             [&](float n) { return fminf(fmaxf(n, -1.f), 1.f) >= tau; });
  }
  cbnd[i] = v;
}

template <int BITS>
__device__ __forceinline__ int nearest_fast(float v, const NearestTable& t) {
  int pos = 0;
#pragma unroll
  for (int step = 1 << (BITS - 1); step >= 1; step >>= 1)
    if (t.tau[pos + step - 1] <= v) pos += step;
  return t.si[pos];
}

// ---------------------------------------------------------------------------
// Emit: one CTA of 256 threads per (kEmitTiles tiles, b, head). KIND 0 = keys,
// 1 = values. Per 16-token block, thread (r, j) = (tid >> 4, tid & 15) takes
// channels 8j..8j+7 of token r with one 16-byte load, so thread order is
// (token, channel) order: a block-wide exclusive scan of the threads' outlier
// counts gives every entry its place in the CSR row. COUNT_ONLY writes the
// block's count into out_ptr[2*(unit*nt_cap + tile) + blk + 1] (prefix-summed
// afterwards into the row pointer over (unit, tile, blk)). Codes go to a
// shared (token, channel) byte tile, from which 128 threads pack the two
// blocks' lane slabs in the decode kernels' fragment-native order.
// ---------------------------------------------------------------------------
constexpr int kEmitThreads = 256;
constexpr int kEmitTiles = 16;

struct EmitArgs {
  const __half* x;
  int64_t B, S, C_full, h0, H, off;
  const float* k_scale;  // keys: [C_full]
  const float* k_zero;
  const float* v_scale;  // values: [B, ld]
  const float* v_zero;
  int64_t ld_stats;
  const Select* sel;     // keys: [B * CL] columns; values: [B * S] rows
  const float* cb;
  int bits;
  uint8_t* codes;
  int64_t nt_cap;
  int32_t* out_ptr;
  uint32_t* out_ent;    // (fp16 value << 16) | (token_in_tile << 7 | channel)
  int64_t nnz_cap;
  __half* sink_out;     // [B, H*128] or null
  __half* dequant_out;  // [B, S, H*128] or null
  // input-space decisions (null: per-element path): outlier bounds per key
  // column [B * CL] / value token [B * S]; code bounds per key channel [CL][16]
  // / value token [B * S][16] (entry 15 = 1 where valid)
  const int4* obnd;
  const int16_t* cbnd;
  const EmitCodebook* ecb;  // the prepared codebook (emit; unused when counting)
};

// Inclusive scan of v over the CTA's 256 threads; also returns the total.
__device__ __forceinline__ int emit_block_scan(int v, int* sh, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  if (lane == 31) sh[w] = v;
  __syncthreads();
  int base = 0;
  total = 0;
#pragma unroll
  for (int k = 0; k < kEmitThreads / 32; ++k) {
    const int x = sh[k];
    base += k < w ? x : 0;
    total += x;
  }
  __syncthreads();  // sh is reused by the next scan
  return base + v;
}

template <int KIND, bool COUNT_ONLY, int BITS>
__global__ void __launch_bounds__(kEmitThreads, 3) emit_kernel(EmitArgs a) {
  __shared__ __align__(16) uint8_t s_code[kTileTokens][kHeadDim];  // codes of the tile
  // code bounds: keys: the head's 128 channels; values: two buffers of a tile's 32 tokens
  __shared__ __align__(16) int16_t s_cbnd[kHeadDim][16];
  __shared__ EmitCodebook s_ec;
  __shared__ int s_scan[kEmitThreads / 32];
  const float* s_cb = s_ec.cb;
  const float* s_cbs = s_ec.cbs;
  const uint8_t* s_cbi = s_ec.cbi;
  const NearestTable& s_nt = s_ec.nt;
  const int64_t b = blockIdx.y, h = blockIdx.z;
  const int tid = threadIdx.x, r = tid >> 4, j = tid & 15;
  const int64_t unit = b * a.H + h;
  const int64_t CL = a.H * kHeadDim;
  const int c0 = 8 * j;                                   // first channel of this thread
  const int64_t cfull0 = (a.h0 + h) * kHeadDim + c0;     // ... in the full row
  const int64_t nt = (a.S + kTileTokens - 1) / kTileTokens;
  const bool with_out = a.nnz_cap >= 0;
  constexpr int ncb = 1 << BITS;
  if (!COUNT_ONLY) {
    load_emit_codebook(a.ecb, &s_ec);
    if (KIND == 0 && a.cbnd) {
      // the head's code bounds, transposed to [bound][channel]: a warp's 16
      // channel chunks then hit distinct bank pairs instead of one bank
      int16_t* t16 = &s_cbnd[0][0];
      for (int i = tid; i < kHeadDim * 16; i += kEmitThreads) {
        const int c = i >> 4, k = i & 15;
        t16[k * kHeadDim + c] = a.cbnd[(h * kHeadDim + c) * 16 + k];
      }
    }
  }
  // keys: this thread's 8 channels' outlier bounds and tie cuts
  int4 kob[8];
  int32_t kcut[8];
  bool kx = KIND == 0 && (!with_out || a.obnd != nullptr) && (COUNT_ONLY || a.cbnd != nullptr);
  if (KIND == 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      kob[e] = make_int4(0, 0, 0, 0);
      kcut[e] = 0;
      if (with_out) {
        kcut[e] = a.sel[b * CL + h * kHeadDim + c0 + e].tie_cut;
        if (a.obnd) kob[e] = a.obnd[b * CL + h * kHeadDim + c0 + e];
        kx = kx && kob[e].x != kNoOrder;
      }
    }
  }
  __syncthreads();
  if (KIND == 0 && !COUNT_ONLY && kx) {
#pragma unroll
    for (int e = 0; e < 8; ++e) kx = kx && (&s_cbnd[0][0])[15 * kHeadDim + c0 + e] == 1;
  }
  const bool fast = COUNT_ONLY ? true : s_nt.fast != 0;
  const int code0 = COUNT_ONLY ? 0 : s_ec.c0;

  // values: a tile's code bounds, 16 bytes per thread for threads 0..63
  const bool vtab = KIND == 1 && !COUNT_ONLY && a.cbnd != nullptr;
  auto load_cb = [&](int64_t tile) {
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    const int64_t t = tile * kTileTokens + (tid >> 1);
    if (tid < 2 * kTileTokens && t < a.S)
      v = reinterpret_cast<const uint4*>(a.cbnd + (b * a.S + t) * 16)[tid & 1];
    return v;
  };
  // this thread's 16-byte input chunk of token r of block blk of a tile
  auto load = [&](int64_t tile, int blk) {
    const int64_t t = tile * kTileTokens + 16 * blk + r;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t < a.S) v = *reinterpret_cast<const uint4*>(a.x + (b * a.S + t) * a.C_full + cfull0);
    return v;
  };
  const int64_t tile_begin = (int64_t)blockIdx.x * kEmitTiles;
  const int64_t tile_end = min(nt, tile_begin + kEmitTiles);
  uint4 nx0 = load(tile_begin, 0), nx1 = load(tile_begin, 1);  // one tile ahead
  uint4 nxb = make_uint4(0u, 0u, 0u, 0u);  // values: the next tile's code bounds
  if (vtab) {
    if (tid < 2 * kTileTokens) reinterpret_cast<uint4*>(&s_cbnd[0][0])[tid] = load_cb(tile_begin);
    __syncthreads();
  }
  for (int64_t tile = tile_begin; tile < tile_end; ++tile) {
    const uint4 cur[2] = {nx0, nx1};
    const int cbuf = (int)((tile - tile_begin) & 1) * kTileTokens;  // values: this tile's rows
    if (tile + 1 < tile_end) {
      nx0 = load(tile + 1, 0);
      nx1 = load(tile + 1, 1);
      if (vtab) nxb = load_cb(tile + 1);
    }
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const int ti = 16 * blk + r;  // token within the tile
      const int64_t t = tile * kTileTokens + ti;
      const bool in = t < a.S;
      const bool is_sink = a.off == 1 && t == 0;
      const bool live = in && !is_sink;
      const uint4 raw = cur[blk];
      const __half* xh = reinterpret_cast<const __half*>(&raw);
      float nval[8];
      uint32_t m8 = 0u;
      uint32_t code_lo = 0u, code_hi = 0u;
      if (live) {
        // the token's outlier bounds and tie cut (values)
        int4 vob = make_int4(0, 0, 0, 0);
        int32_t vcut = 0;
        bool xs = KIND == 0 ? kx : false;
        if (KIND == 1) {
          if (with_out) vcut = a.sel[b * a.S + t].tie_cut;
          xs = (!with_out || a.obnd != nullptr) &&
               (COUNT_ONLY || (a.cbnd != nullptr && s_cbnd[cbuf + ti][15] == 1));
          if (xs && with_out) {
            vob = a.obnd[b * a.S + t];
            xs = vob.x != kNoOrder;
          }
        }
        if (xs && fast && finite8(raw)) {
          // decisions by the input's order against the precomputed bounds
          const int16_t* crow = KIND == 0 ? nullptr : &s_cbnd[cbuf + ti][0];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint16_t hb = __half_as_ushort(xh[e]);
            const int o = ord16(hb);
            const bool out = with_out && (KIND == 0 ? out_by_order(o, kob[e], (int32_t)(t - a.off), kcut[e])
                                                    : out_by_order(o, vob, (int32_t)(cfull0 + e), vcut));
            if (out) m8 |= 1u << e;
            if (!COUNT_ONLY) {
              const int code =
                  out ? code0
                      : (int)s_nt.si[KIND == 0
                                         ? pos_by_order<BITS>(o, &s_cbnd[0][0] + c0 + e, kHeadDim)
                                         : pos_by_order<BITS>(o, crow)];
              if (e < 4) code_lo |= (uint32_t)code << (8 * e);
              else code_hi |= (uint32_t)code << (8 * (e - 4));
            }
          }
        } else {
          // per element: IEEE normalization, selection and nearest centroid
          const Select sl = KIND == 0 ? Select{} : (with_out ? a.sel[b * a.S + t] : Select{});
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float zz = KIND == 0 ? a.k_zero[cfull0 + e] : a.v_zero[b * a.ld_stats + t];
            const float ss = KIND == 0 ? a.k_scale[cfull0 + e] : a.v_scale[b * a.ld_stats + t];
            const float n = normalize(__half2float(xh[e]), zz, ss);
            bool out = false;
            if (with_out) {
              const Select se = KIND == 0 ? a.sel[b * CL + h * kHeadDim + c0 + e] : sl;
              out = selected(abs_bits(n), KIND == 0 ? (int32_t)(t - a.off) : (int32_t)(cfull0 + e), se);
            }
            if (out) m8 |= 1u << e;
            if (!COUNT_ONLY) {
              const float dense = out ? 0.f : fminf(fmaxf(n, -1.f), 1.f);
              const int code = fast ? nearest_fast<BITS>(dense, s_nt)
                                    : nearest_centroid_sorted(dense, s_cbs, s_cbi, ncb);
              if (e < 4) code_lo |= (uint32_t)code << (8 * e);
              else code_hi |= (uint32_t)code << (8 * (e - 4));
            }
          }
        }
        // outlier entries and the optional dequantized output need n and dq
        if (!COUNT_ONLY && (m8 || a.dequant_out)) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const bool out = (m8 >> e) & 1u;
            if (!out && !a.dequant_out) continue;
            const float zz = KIND == 0 ? a.k_zero[cfull0 + e] : a.v_zero[b * a.ld_stats + t];
            const float ss = KIND == 0 ? a.k_scale[cfull0 + e] : a.v_scale[b * a.ld_stats + t];
            const int code = (int)(((e < 4 ? code_lo : code_hi) >> (8 * (e & 3))) & 0xffu);
            const float n = out ? normalize(__half2float(xh[e]), zz, ss) : 0.f;
            const float dq = dequant_ref(s_cb[code], n, ss, zz);
            nval[e] = dq;  // the entry holds the dequantized value
            if (a.dequant_out)
              a.dequant_out[(b * a.S + t) * CL + h * kHeadDim + c0 + e] = __float2half_rn(dq);
          }
        }
      } else if (!COUNT_ONLY && a.dequant_out && in) {  // the sink token: its input
        *reinterpret_cast<uint4*>(a.dequant_out + (b * a.S + t) * CL + h * kHeadDim + c0) = raw;
      }
      if (!COUNT_ONLY) {
        *reinterpret_cast<uint2*>(&s_code[ti][c0]) = make_uint2(code_lo, code_hi);
        if (a.sink_out && is_sink)
          *reinterpret_cast<uint4*>(a.sink_out + b * CL + h * kHeadDim + c0) = raw;
      }
      const int cnt = __popc(m8);
      int total;
      const int incl = emit_block_scan(cnt, s_scan, total);
      const int64_t row = 2 * (unit * a.nt_cap + tile) + blk;
      if (COUNT_ONLY) {
        if (tid == 0) a.out_ptr[row + 1] = total;
      } else if (m8) {
        int64_t e_idx = (int64_t)a.out_ptr[row] + incl - cnt;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if ((m8 >> e) & 1u) {
            if (e_idx < a.nnz_cap) a.out_ent[e_idx] = outlier_entry(ti, c0 + e, nval[e]);
            ++e_idx;
          }
        }
      }
    }
    if (COUNT_ONLY) continue;
    __syncthreads();  // the tile's codes are in s_code
    // Slab store: thread (slab, half) = (tid >> 1, tid & 1) packs slots
    // 16*half .. 16*half+15 of the slab of (block, lane) = (slab >> 5, slab & 31).
    if (tid < 128) {
      const int slab = tid >> 1, half = tid & 1;
      const int blk = slab >> 5, lane = slab & 31;
      const int g = lane >> 2, cc = lane & 3;
      uint32_t wd[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int qq = 0; qq < 16; ++qq) {
        const int q = 16 * half + qq;
        int ta, ca, tb, cb2;
        if (KIND == 0) {  // keys: token 16*blk + g + 8*(q&1), RoPE pair 4*(q>>1) + cc
          ta = tb = 16 * blk + g + 8 * (q & 1);
          ca = 4 * (q >> 1) + cc;
          cb2 = ca + 64;
        } else {          // values: channel 16*(q>>2) + g + 8*(q&1), tokens (t, t+1)
          ca = cb2 = 16 * (q >> 2) + g + 8 * (q & 1);
          ta = 16 * blk + 2 * cc + 8 * ((q >> 1) & 1);
          tb = ta + 1;
        }
        const uint32_t pair = (uint32_t)s_code[ta][ca] | ((uint32_t)s_code[tb][cb2] << BITS);
        const int bit = 2 * BITS * qq;
        wd[bit >> 5] |= pair << (bit & 31);
        if ((bit & 31) + 2 * BITS > 32) wd[(bit >> 5) + 1] |= pair >> (32 - (bit & 31));
      }
      // The block is stored structure-of-arrays: bytes 0..15 of every lane's
      // slab (512 B), then its remaining 8*BITS-16 bytes, so that the decode
      // kernels' per-lane copies are coalesced. This half covers slab words
      // half*BITS .. half*BITS + BITS - 1.
      uint8_t* blk_base = a.codes + (unit * a.nt_cap + tile) * (int64_t)tile_bytes(BITS) +
                          blk * (256 * BITS);
#pragma unroll
      for (int k = 0; k < BITS; ++k) {
        const int wb = 4 * (half * BITS + k);  // byte offset in the slab
        uint8_t* dst = wb < 16 ? blk_base + lane * 16 + wb
                               : blk_base + 512 + lane * (8 * BITS - 16) + (wb - 16);
        *reinterpret_cast<uint32_t*>(dst) = wd[k];
      }
    }
    // values: the next tile's code bounds into the other buffer (nobody reads it now)
    if (vtab && tid < 2 * kTileTokens && tile + 1 < tile_end)
      reinterpret_cast<uint4*>(&s_cbnd[kTileTokens - cbuf][0])[tid] = nxb;
    __syncthreads();  // s_code is rewritten by the next tile; the bounds are visible
  }
}

// Clears code tiles nt .. nt_cap-1 of every unit (so stale codes never reach
// the decode kernels). grid-stride over 16-byte words.
__global__ void clear_tail_tiles_kernel(uint8_t* __restrict__ codes, int64_t units, int64_t nt,
                                        int64_t nt_cap, int64_t tb) {
  const int64_t per_unit = (nt_cap - nt) * tb / 16;
  const int64_t total = units * per_unit;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t u = i / per_unit, w = i % per_unit;
    reinterpret_cast<uint4*>(codes + (u * nt_cap + nt) * tb)[w] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Exclusive scan of the per-row counts stored at ptr[1..n] (ptr[0] = 0) into
// the CSR row pointer, and the total nnz; n is the number of rows. Three
// launches and no scratch: (1) every chunk of kScanChunk counts is scanned in
// place (inclusive, local); (2) one CTA turns the chunk totals (each chunk's
// last element) into their final values; (3) every chunk but the first adds
// the final value of the previous chunk's last element to its other elements.
constexpr int kScanThreads = 1024, kScanPer = 4, kScanChunk = kScanThreads * kScanPer;

__device__ __forceinline__ int64_t block_incl_scan(int64_t v, int64_t* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  if (lane == 31) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    int64_t x = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int64_t o = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += o;
    }
    sh[lane] = x;
  }
  __syncthreads();
  const int64_t r = v + (w > 0 ? sh[w - 1] : 0);
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kScanThreads) scan_chunks_kernel(int32_t* __restrict__ ptr, int64_t n) {
  __shared__ int64_t sh[32];
  const int64_t i0 = (int64_t)blockIdx.x * kScanChunk + (int64_t)threadIdx.x * kScanPer;
  int32_t v[kScanPer];
  int64_t sum = 0;
#pragma unroll
  for (int k = 0; k < kScanPer; ++k) {
    v[k] = i0 + k < n ? ptr[1 + i0 + k] : 0;
    sum += v[k];
  }
  int64_t run = block_incl_scan(sum, sh) - sum;
#pragma unroll
  for (int k = 0; k < kScanPer; ++k) {
    run += v[k];
    if (i0 + k < n) ptr[1 + i0 + k] = (int32_t)run;
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_totals_kernel(int32_t* __restrict__ ptr, int64_t n,
                                                                  int64_t* __restrict__ nnz_out) {
  __shared__ int64_t sh[32];
  const int64_t nb = (n + kScanChunk - 1) / kScanChunk;
  int64_t carry = 0;
  for (int64_t c0 = 0; c0 < nb; c0 += kScanThreads) {
    const int64_t c = c0 + threadIdx.x;
    const int64_t last = c < nb ? min(n, (c + 1) * kScanChunk) : 0;  // index (1-based) of the chunk's last count
    const int64_t tot = c < nb ? ptr[last] : 0;
    const int64_t incl = block_incl_scan(tot, sh);
    if (c < nb) ptr[last] = (int32_t)(carry + incl);
    if (threadIdx.x == kScanThreads - 1) sh[0] = incl;  // this batch's total
    __syncthreads();
    carry += sh[0];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    ptr[0] = 0;
    if (nnz_out) *nnz_out = carry;
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_offsets_kernel(int32_t* __restrict__ ptr, int64_t n) {
  const int64_t c = (int64_t)blockIdx.x + 1;  // chunk 0 needs no offset
  const int32_t off = ptr[c * kScanChunk];    // final value of the previous chunk's last count
  const int64_t last = min(n, (c + 1) * kScanChunk);
  for (int64_t i = c * kScanChunk + 1 + threadIdx.x; i < last; i += kScanThreads) ptr[i] += off;
}

static void scan_counts(int32_t* ptr, int64_t n, int64_t* nnz_out, cudaStream_t st) {
  const int64_t nb = (n + kScanChunk - 1) / kScanChunk;
  scan_chunks_kernel<<<(unsigned)nb, kScanThreads, 0, st>>>(ptr, n);
  scan_totals_kernel<<<1, kScanThreads, 0, st>>>(ptr, n, nnz_out);
  if (nb > 1) scan_offsets_kernel<<<(unsigned)(nb - 1), kScanThreads, 0, st>>>(ptr, n);
}

__global__ void init_select_kernel(Select* __restrict__ sel, int64_t n, int32_t k) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    Select s;
    s.thr = 0;
    s.kleft = k;
    s.tie_cut = 0x7fffffff;
    s.ties = 0;
    sel[i] = s;
  }
}

__global__ void zero_i32_kernel(int32_t* __restrict__ p, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = 0;
}

// Workspace layout.
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// keys: selections [B*CL], histograms [B*CL][256] (then the tie counts),
// outlier bounds [B*CL] int4, code bounds [CL][16] int16
inline size_t key_ws_bytes(int64_t B, int64_t n_heads) {
  const int64_t ncols = B * n_heads * kHeadDim;
  return align256(ncols * sizeof(Select)) + align256(ncols * 256 * sizeof(uint32_t)) +
         align256(ncols * sizeof(int4)) + align256(n_heads * kHeadDim * 16 * sizeof(int16_t)) +
         align256(sizeof(EmitCodebook));
}
inline int4* key_obnd(void* ws, int64_t B, int64_t n_heads) {
  const int64_t ncols = B * n_heads * kHeadDim;
  return reinterpret_cast<int4*>((char*)ws + align256(ncols * sizeof(Select)) +
                                 align256(ncols * 256 * sizeof(uint32_t)));
}
inline int16_t* key_cbnd(void* ws, int64_t B, int64_t n_heads) {
  const int64_t ncols = B * n_heads * kHeadDim;
  return reinterpret_cast<int16_t*>((char*)key_obnd(ws, B, n_heads) + align256(ncols * sizeof(int4)));
}
inline EmitCodebook* key_ecb(void* ws, int64_t B, int64_t n_heads) {
  return reinterpret_cast<EmitCodebook*>(
      (char*)key_cbnd(ws, B, n_heads) + align256(n_heads * kHeadDim * 16 * sizeof(int16_t)));
}
// values: selections [B*S], outlier bounds [B*S] int4, code bounds [B*S][16] int16
inline size_t value_ws_bytes(int64_t B, int64_t S) {
  return align256((size_t)B * S * sizeof(Select)) + align256((size_t)B * S * sizeof(int4)) +
         align256((size_t)B * S * 16 * sizeof(int16_t)) + align256(sizeof(EmitCodebook));
}
inline int4* value_obnd(void* ws, int64_t B, int64_t S) {
  return reinterpret_cast<int4*>((char*)ws + align256((size_t)B * S * sizeof(Select)));
}
inline int16_t* value_cbnd(void* ws, int64_t B, int64_t S) {
  return reinterpret_cast<int16_t*>((char*)value_obnd(ws, B, S) +
                                    align256((size_t)B * S * sizeof(int4)));
}
inline EmitCodebook* value_ecb(void* ws, int64_t B, int64_t S) {
  return reinterpret_cast<EmitCodebook*>((char*)value_cbnd(ws, B, S) +
                                         align256((size_t)B * S * 16 * sizeof(int16_t)));
}

inline bool bits_ok(int bits) { return bits >= 2 && bits <= 4; }

// Threads of value_plan_kernel for a row of C_full channels (16 per thread).
inline int plan_threads(int64_t C_full) {
  return (int)((C_full + kPlanEPT * 32 - 1) / (kPlanEPT * 32)) * 32;
}

inline dim3 emit_grid(int64_t S, int64_t B, int64_t n_heads) {
  const int64_t nt = (S + kTileTokens - 1) / kTileTokens;
  return dim3((unsigned)((nt + kEmitTiles - 1) / kEmitTiles), (unsigned)B, (unsigned)n_heads);
}

template <int KIND>
static void launch_emit(const EmitArgs& ea, bool count_only, cudaStream_t st) {
  const dim3 grid = emit_grid(ea.S, ea.B, ea.H);
  if (count_only) {
    emit_kernel<KIND, true, 2><<<grid, kEmitThreads, 0, st>>>(ea);
    return;
  }
  switch (ea.bits) {
    case 2: emit_kernel<KIND, false, 2><<<grid, kEmitThreads, 0, st>>>(ea); break;
    case 3: emit_kernel<KIND, false, 3><<<grid, kEmitThreads, 0, st>>>(ea); break;
    default: emit_kernel<KIND, false, 4><<<grid, kEmitThreads, 0, st>>>(ea); break;
  }
}

// Clears the code tiles after the block's last tile, for every unit.
static void clear_tail(uint8_t* codes, int64_t units, int64_t nt, int64_t nt_cap, int bits,
                       cudaStream_t st) {
  if (nt_cap <= nt) return;
  const int64_t words = units * (nt_cap - nt) * tile_bytes(bits) / 16;
  clear_tail_tiles_kernel<<<grid_for(words, 256), 256, 0, st>>>(codes, units, nt, nt_cap,
                                                                tile_bytes(bits));
}

}  // namespace kvq

extern "C" size_t kvq_quantize_keys_workspace(int64_t B, int64_t S, int64_t n_heads) {
  (void)S;
  return kvq::key_ws_bytes(B, n_heads);
}

extern "C" size_t kvq_quantize_values_workspace(int64_t B, int64_t S, int64_t n_heads) {
  (void)n_heads;
  return kvq::value_ws_bytes(B, S);
}

namespace kvq {

static int check_block(const char* what, int64_t B, int64_t S, int64_t C_full, int64_t h0,
                       int64_t n_heads, int64_t nt_cap) {
  if (B < 1 || S < 1 || n_heads < 1 || h0 < 0 || C_full < (h0 + n_heads) * kHeadDim) {
    set_error("%s: invalid shape B=%lld S=%lld C_full=%lld heads [%lld, %lld)", what,
              (long long)B, (long long)S, (long long)C_full, (long long)h0,
              (long long)(h0 + n_heads));
    return KVQ_ERR_INVALID;
  }
  if (nt_cap * kTileTokens < S) {
    set_error("%s: nt_cap=%lld tiles cannot hold S=%lld tokens", what, (long long)nt_cap,
              (long long)S);
    return KVQ_ERR_INVALID;
  }
  if (S > (1LL << 30) || B * n_heads * nt_cap >= (1LL << 31)) {
    set_error("%s: block too large", what);
    return KVQ_ERR_INVALID;
  }
  return KVQ_OK;
}

// The emit kernels stage a tile's inputs with 16-byte loads.
static int check_x(const char* what, const void* x, int64_t C_full) {
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || C_full % 8 != 0) {
    set_error("%s: the input must be 16-byte aligned with C_full a multiple of 8", what);
    return KVQ_ERR_INVALID;
  }
  return KVQ_OK;
}

}  // namespace kvq

extern "C" int kvq_quantize_keys_plan(const void* k, int64_t B, int64_t S, int64_t C_full,
                                      int64_t h0, int64_t n_heads, const float* scale,
                                      const float* zero, double outlier_ratio, int sink,
                                      int32_t* out_ptr, int64_t nt_cap, int64_t* nnz_out,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_block("quantize_keys_plan", B, S, C_full, h0, n_heads, nt_cap);
  if (!rc) rc = check_x("quantize_keys_plan", k, C_full);
  if (rc) return rc;
  if (workspace_bytes < key_ws_bytes(B, n_heads) || !workspace) {
    set_error("quantize_keys_plan: workspace too small (%zu < %zu)", workspace_bytes,
              key_ws_bytes(B, n_heads));
    return KVQ_ERR_INVALID;
  }
  cudaStream_t st = as_stream(stream);
  const int64_t CL = n_heads * kHeadDim, ncols = B * CL;
  Select* sel = reinterpret_cast<Select*>(workspace);
  uint32_t* hist = reinterpret_cast<uint32_t*>((char*)workspace + align256(ncols * sizeof(Select)));
  KeyShape ks{(const __half*)k, B, S, C_full, h0 * kHeadDim, CL, (sink && S > 1) ? 1 : 0,
              scale, zero};
  const int64_t n_rest = S - ks.off;
  const bool outliers = outlier_ratio > 0;
  const int64_t kk = outliers ? outlier_count(n_rest, outlier_ratio) : 0;
  init_select_kernel<<<(unsigned)((ncols + 255) / 256), 256, 0, st>>>(sel, ncols, (int32_t)kk);
  if (outliers) {
    cudaMemsetAsync(hist, 0, ncols * 256 * sizeof(uint32_t), st);
    const int64_t rows_per_block = 4096;
    dim3 hg((unsigned)(CL / kHistCols), (unsigned)B,
            (unsigned)((n_rest + rows_per_block - 1) / rows_per_block));
    for (int shift = 24; shift >= 0; shift -= 8) {
      key_hist_kernel<<<hg, 256, 0, st>>>(ks, shift, sel, hist, rows_per_block);
      key_select_kernel<<<(unsigned)((ncols + 127) / 128), 128, 0, st>>>(sel, hist, ncols, shift);
    }
    // tie counts per (column, row block) in the (now zero) histogram memory
    const int64_t trb = tie_rows_per_block(n_rest);
    const int nrb = (int)((n_rest + trb - 1) / trb);
    int32_t* tcounts = reinterpret_cast<int32_t*>(hist);
    key_ties_count_kernel<<<dim3((unsigned)(CL / kHistCols), (unsigned)B, (unsigned)nrb), 256, 0,
                            st>>>(ks, sel, tcounts, trb, nrb);
    key_ties_find_kernel<<<(unsigned)((ncols + 7) / 8), 256, 0, st>>>(ks, sel, tcounts, trb, nrb,
                                                                      ncols);
    // each column's outlier decisions as bounds on the input order
    key_out_bounds_kernel<<<(unsigned)((ncols * 4 + 255) / 256), 256, 0, st>>>(
        ks, sel, key_obnd(workspace, B, n_heads), ncols);
  }
  // Outlier counts per (unit, tile, block), then the row pointer.
  const int64_t nrows = 2 * B * n_heads * nt_cap;  // (unit, tile, 16-token block)
  zero_i32_kernel<<<grid_for(nrows + 1, 256), 256, 0, st>>>(out_ptr, nrows + 1);
  EmitArgs ea{};
  ea.x = ks.k; ea.B = B; ea.S = S; ea.C_full = C_full; ea.h0 = h0; ea.H = n_heads;
  ea.off = ks.off; ea.k_scale = scale; ea.k_zero = zero; ea.sel = sel; ea.bits = 2;
  ea.nt_cap = nt_cap; ea.out_ptr = out_ptr; ea.nnz_cap = outliers ? 0 : -1;
  ea.cb = nullptr;  // COUNT_ONLY never reads the codebook
  ea.obnd = outliers ? key_obnd(workspace, B, n_heads) : nullptr;
  launch_emit<0>(ea, true, st);
  scan_counts(out_ptr, nrows, nnz_out, st);
  return check_launch("quantize_keys_plan");
}

extern "C" int kvq_quantize_keys_emit(const void* k, int64_t B, int64_t S, int64_t C_full,
                                      int64_t h0, int64_t n_heads, const float* scale,
                                      const float* zero, const float* codebook, int bits,
                                      double outlier_ratio, int sink, uint8_t* codes,
                                      int64_t nt_cap, const int32_t* out_ptr, uint32_t* out_ent,
                                      int64_t nnz_cap, void* sink_out,
                                      void* dequant_out, const void* workspace,
                                      size_t workspace_bytes, void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_block("quantize_keys_emit", B, S, C_full, h0, n_heads, nt_cap);
  if (!rc) rc = check_x("quantize_keys_emit", k, C_full);
  if (rc) return rc;
  if (!bits_ok(bits)) {
    set_error("quantize_keys_emit: bits must be 2, 3 or 4 (got %d)", bits);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (workspace_bytes < key_ws_bytes(B, n_heads) || !workspace) {
    set_error("quantize_keys_emit: workspace too small");
    return KVQ_ERR_INVALID;
  }
  cudaStream_t st = as_stream(stream);
  const int64_t nt = (S + kTileTokens - 1) / kTileTokens;
  // Tiles beyond the block are cleared so stale codes never reach the decode kernels.
  clear_tail(codes, B * n_heads, nt, nt_cap, bits, st);
  EmitArgs ea{};
  ea.x = (const __half*)k; ea.B = B; ea.S = S; ea.C_full = C_full; ea.h0 = h0;
  ea.H = n_heads; ea.off = (sink && S > 1) ? 1 : 0; ea.k_scale = scale; ea.k_zero = zero;
  ea.sel = reinterpret_cast<const Select*>(workspace); ea.cb = codebook; ea.bits = bits;
  ea.codes = codes; ea.nt_cap = nt_cap; ea.out_ptr = const_cast<int32_t*>(out_ptr);
  ea.out_ent = out_ent;
  ea.nnz_cap = outlier_ratio > 0 ? nnz_cap : -1;
  ea.sink_out = (__half*)sink_out; ea.dequant_out = (__half*)dequant_out;
  // code decisions of the head range's channels as bounds on the input order
  void* ws = const_cast<void*>(workspace);
  const int64_t CL = n_heads * kHeadDim;
  codebook_setup_kernel<<<1, 32, 0, st>>>(codebook, bits, key_ecb(ws, B, n_heads));
  code_bounds_kernel<<<(unsigned)((CL * 16 + 255) / 256), 256, 0, st>>>(
      zero + h0 * kHeadDim, scale + h0 * kHeadDim, CL, CL, 0, key_ecb(ws, B, n_heads), bits,
      key_cbnd(ws, B, n_heads));
  ea.ecb = key_ecb(ws, B, n_heads);
  ea.obnd = outlier_ratio > 0 ? key_obnd(ws, B, n_heads) : nullptr;
  ea.cbnd = key_cbnd(ws, B, n_heads);
  launch_emit<0>(ea, false, st);
  return check_launch("quantize_keys_emit");
}

extern "C" int kvq_quantize_values_plan(const void* v, int64_t B, int64_t S, int64_t C_full,
                                        int64_t h0, int64_t n_heads, double outlier_ratio,
                                        int sink, float* v_scale, float* v_zero,
                                        int64_t ld_stats, int32_t* out_ptr, int64_t nt_cap,
                                        int64_t* nnz_out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_block("quantize_values_plan", B, S, C_full, h0, n_heads, nt_cap);
  if (!rc) rc = check_x("quantize_values_plan", v, C_full);
  if (rc) return rc;
  if (C_full > kValRowMax) {
    set_error("quantize_values_plan: C=%lld channels exceed %d", (long long)C_full, kValRowMax);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (ld_stats < S) {
    set_error("quantize_values_plan: ld_stats=%lld < S=%lld", (long long)ld_stats, (long long)S);
    return KVQ_ERR_INVALID;
  }
  if (workspace_bytes < value_ws_bytes(B, S) || !workspace) {
    set_error("quantize_values_plan: workspace too small");
    return KVQ_ERR_INVALID;
  }
  cudaStream_t st = as_stream(stream);
  Select* sel = reinterpret_cast<Select*>(workspace);
  const int64_t off = (sink && S > 1) ? 1 : 0;
  const int64_t n_rest = S - off;
  const bool outliers = outlier_ratio > 0;
  const int64_t kv = outliers ? outlier_count(C_full, outlier_ratio) : 0;
  const int64_t nrows = 2 * B * n_heads * nt_cap;  // (unit, tile, 16-token block)
  zero_i32_kernel<<<grid_for(nrows + 1, 256), 256, 0, st>>>(out_ptr, nrows + 1);
  if (B * n_rest > 0) {
    // per-token stats, selections and the outlier counts of each CSR row
    const size_t smem = C_full * sizeof(uint32_t);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(value_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
    value_plan_kernel<<<(unsigned)(B * n_rest), plan_threads(C_full), smem, st>>>(
        (const __half*)v, B, S, C_full, off, kv, v_scale, v_zero, ld_stats, sel,
        outliers ? out_ptr : nullptr, h0, n_heads, nt_cap);
    if (outliers)  // each token's outlier decisions as bounds on the input order
      value_out_bounds_kernel<<<(unsigned)((B * S * 4 + 255) / 256), 256, 0, st>>>(
          v_zero, v_scale, ld_stats, sel, B, S, off, value_obnd(workspace, B, S));
  }
  if (off) {  // the sink token carries no stats
    for (int64_t b = 0; b < B; ++b) {
      if (cudaMemsetAsync(v_scale + b * ld_stats, 0, sizeof(float), st) != cudaSuccess ||
          cudaMemsetAsync(v_zero + b * ld_stats, 0, sizeof(float), st) != cudaSuccess)
        return check_launch("quantize_values_plan");
    }
  }
  scan_counts(out_ptr, nrows, nnz_out, st);
  return check_launch("quantize_values_plan");
}

extern "C" int kvq_quantize_values_emit(const void* v, int64_t B, int64_t S, int64_t C_full,
                                        int64_t h0, int64_t n_heads, const float* codebook,
                                        int bits, double outlier_ratio, int sink,
                                        const float* v_scale, const float* v_zero,
                                        int64_t ld_stats, uint8_t* codes, int64_t nt_cap,
                                        const int32_t* out_ptr, uint32_t* out_ent,
                                        int64_t nnz_cap, void* sink_out,
                                        void* dequant_out, const void* workspace,
                                        size_t workspace_bytes, void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_block("quantize_values_emit", B, S, C_full, h0, n_heads, nt_cap);
  if (!rc) rc = check_x("quantize_values_emit", v, C_full);
  if (rc) return rc;
  if (!bits_ok(bits)) {
    set_error("quantize_values_emit: bits must be 2, 3 or 4 (got %d)", bits);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (workspace_bytes < value_ws_bytes(B, S) || !workspace || ld_stats < S) {
    set_error("quantize_values_emit: workspace too small or ld_stats < S");
    return KVQ_ERR_INVALID;
  }
  cudaStream_t st = as_stream(stream);
  const int64_t nt = (S + kTileTokens - 1) / kTileTokens;
  clear_tail(codes, B * n_heads, nt, nt_cap, bits, st);
  EmitArgs ea{};
  ea.x = (const __half*)v; ea.B = B; ea.S = S; ea.C_full = C_full; ea.h0 = h0;
  ea.H = n_heads; ea.off = (sink && S > 1) ? 1 : 0; ea.v_scale = v_scale; ea.v_zero = v_zero;
  ea.ld_stats = ld_stats; ea.sel = reinterpret_cast<const Select*>(workspace);
  ea.cb = codebook; ea.bits = bits; ea.codes = codes; ea.nt_cap = nt_cap;
  ea.out_ptr = const_cast<int32_t*>(out_ptr); ea.out_ent = out_ent;
  ea.nnz_cap = outlier_ratio > 0 ? nnz_cap : -1;
  ea.sink_out = (__half*)sink_out; ea.dequant_out = (__half*)dequant_out;
  // code decisions of every token as bounds on the input order
  void* ws = const_cast<void*>(workspace);
  codebook_setup_kernel<<<1, 32, 0, st>>>(codebook, bits, value_ecb(ws, B, S));
  code_bounds_kernel<<<(unsigned)((B * S * 16 + 255) / 256), 256, 0, st>>>(
      v_zero, v_scale, B * S, S, ld_stats, value_ecb(ws, B, S), bits, value_cbnd(ws, B, S));
  ea.ecb = value_ecb(ws, B, S);
  ea.obnd = outlier_ratio > 0 ? value_obnd(ws, B, S) : nullptr;
  ea.cbnd = value_cbnd(ws, B, S);
  launch_emit<1>(ea, false, st);
  return check_launch("quantize_values_emit");
}
