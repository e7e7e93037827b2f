// Decode attention over the packed quantized cache.
//
// Key kernel: score[b,hq,t] = q . RoPE_t(Khat_t), Khat = (cb[code] + o) * s + z
// per channel (kvquant/quant/kv_quantizer.py:89), rotate-half RoPE with fp32
// angles fl(t * inv_freq) (kvquant/kernels/rope_fused.py:6-12). Per RoPE pair
// (channels p, p+64) with code values L1, L2:
//   X = L1*(s1 q1) + L2*(s2 q2) + (z1 q1 + z2 q2)
//   Y = L1*(s1 q2) - L2*(s2 q1) + (z1 q2 - z2 q1)
//   score += cos(t th_p) * X + sin(t th_p) * Y
// The per-(query head, pair) constants are built once per CTA; cos/sin once per
// (token, pair) per CTA and reused by every head the CTA owns; the code->value
// LUT is a conflict-free shared-memory pair table; X and Y use the sm_100
// fp16 x fp16 + fp32 FMA; outliers are added from the tile-CSR afterwards.
//
// Value kernel: out[b,hq,:] = sum_t p_t * (s_t * (cb[code] + o) + z_t) with the
// per-token scale s_t / zero z_t over all channels (kv_quantizer.py:103-117).
#pragma once
#include "kvq_common.cuh"

namespace kvq {

// ---------------------------------------------------------------------------
// cos/sin of the fp32 angle a = fl(t * f): reduction by 2*pi in fp64 (exact to
// ~1e-9 rad for |a| < 2^24), then the hardware sin/cos on [-pi, pi].
// ---------------------------------------------------------------------------
__device__ __forceinline__ void rope_cos_sin(int64_t t, float f, float& c, float& s) {
  const float a = __fmul_rn((float)t, f);
  const double ad = (double)a;
  const double k = rint(ad * 0.15915494309189535);  // 1 / (2 pi)
  double r = fma(-k, 6.283185307179586, ad);        // 2 pi (high part)
  r = fma(-k, 2.4492935982947064e-16, r);           // 2 pi - high part
  __sincosf((float)r, &s, &c);
}

// Exponent e with m <= 2^e (0 for m == 0), clamped to [-100, 100] so that
// 2^e and 2^-e stay finite fp32 numbers: a slot whose largest magnitude is
// below 2^-100 (e.g. softmax weights that underflowed) contributes nothing
// measurable, and scaling it by at most 2^114 cannot overflow.
__device__ __forceinline__ int pow2_exponent(float m) {
  int ex = 0;
  if (m > 0.f) frexpf(m, &ex);
  return ex < -100 ? -100 : (ex > 100 ? 100 : ex);
}

// Shared-memory pair LUT: entry v (a pair of codes, low code in the low bits)
// holds half2(cb[lo], cb[hi]); each of the 32 lanes owns a copy at byte
// (v << 8) | (lane << 2), so a warp's 32 lookups hit 32 distinct banks.
// Bytes 128..255 of every 256-byte row are free for other data.
template <int BITS>
struct PairLut {
  static constexpr int kEntries = 1 << (2 * BITS);
  static constexpr int kBytes = kEntries * 256;
  __device__ static void build(uint8_t* smem, const float* cb) {
    constexpr int mask = (1 << BITS) - 1;
    for (int idx = threadIdx.x; idx < kEntries * 32; idx += blockDim.x) {
      const int v = idx >> 5, lane = idx & 31;
      const uint32_t h = half2_bits(cb[v & mask], cb[v >> BITS]);
      *reinterpret_cast<uint32_t*>(smem + (v << 8) + (lane << 2)) = h;
    }
  }
  // Byte address (relative to the table) of pair m of the slab for this lane.
  __device__ static __forceinline__ uint32_t addr(const uint32_t* slab, int m, uint32_t lane4) {
    if (BITS == 4) {
      // byte m of the slab -> bits 8..15; lane*4 -> bits 0..7 (one PRMT)
      const uint32_t w = slab[m >> 2];
      const uint32_t sel = 0x1100u | ((4u + (m & 3)) << 4);
      return prmt(lane4, w, sel);
    } else {
      return (slab_pair<BITS>(slab, m) << 8) | lane4;
    }
  }
};

template <int BITS>
struct CodeSlab {
  static constexpr int kWords = BITS;  // 4*BITS bytes
  uint32_t w[4];
  __device__ __forceinline__ void load(const uint8_t* p) {
    if (BITS == 4) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if (BITS == 2) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = v.x; w[1] = v.y; w[2] = 0; w[3] = 0;
    } else {
      const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
      w[0] = __ldg(q); w[1] = __ldg(q + 1); w[2] = __ldg(q + 2); w[3] = 0;
    }
  }
};

// Per-(slot, pair) key constants, 16 bytes: fp16 {P1, P2} {Q1, Q2}, fp32 OX, OY
// (all divided by the slot's power-of-two sigma).
struct KeyConst {
  uint32_t p12, q12;
  float ox, oy;
};

struct KeyArgs {
  const uint8_t* codes;
  const __half* out_vals;
  const uint16_t* out_pos;
  const int32_t* out_ptr;
  const float* k_scale;  // [H*128] local channels
  const float* k_zero;
  const __half* k_sink;  // [B, H*128] or null
  const float* cb;
  const __half* q;       // [B, H*G, 128]
  const float* inv_freq; // [64]
  int64_t B, H, G, T, nt_cap;
  float* scores;         // [B, H*G, T]
  int units_per_group, n_groups;
  int64_t n_items;       // tile pairs * groups
};

constexpr int kKeyThreads = 128;
constexpr int kMaxSlots = 32;  // query heads per group

template <int BITS>
__host__ __device__ constexpr int key_const_offset() {
  return BITS == 4 ? 0 : PairLut<BITS>::kBytes;  // 4-bit: constants live in LUT holes
}
template <int BITS>
__host__ __device__ constexpr int key_smem_bytes() {
  return (BITS == 4 ? PairLut<4>::kBytes : PairLut<BITS>::kBytes + kMaxSlots * kPairs * 16) +
         kMaxSlots * 64 * 4 + kMaxSlots * 4;
}

// Address of the constants of (slot, pair p) inside shared memory.
template <int BITS>
__device__ __forceinline__ KeyConst* key_const(uint8_t* smem, int slot, int p) {
  if (BITS == 4) {
    // slot*64 + p -> row r of the LUT (0..2047 of 16-byte cells); row = idx/8, cell = idx%8
    const int idx = slot * kPairs + p;
    return reinterpret_cast<KeyConst*>(smem + ((idx >> 3) << 8) + 128 + ((idx & 7) << 4));
  }
  return reinterpret_cast<KeyConst*>(smem + key_const_offset<BITS>()) + slot * kPairs + p;
}

template <int BITS, int G>
__global__ void __launch_bounds__(kKeyThreads) key_scores_kernel(KeyArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* lut = smem;
  constexpr int kConstEnd = BITS == 4 ? PairLut<4>::kBytes : PairLut<BITS>::kBytes + kMaxSlots * kPairs * 16;
  float* sc = reinterpret_cast<float*>(smem + kConstEnd);  // [slots][64 tokens]
  float* sigma = sc + kMaxSlots * 64;                      // [slots]

  const int j = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lane4 = (uint32_t)lane << 2;
  PairLut<BITS>::build(lut, a.cb);

  const int64_t nt = (a.T + kTileTokens - 1) / kTileTokens;
  const int64_t n_pairs = (nt + 1) / 2;
  const int UG = a.units_per_group;
  const int slots = UG * G;
  // Static contiguous split of the (group-major) work list.
  const int64_t w0 = a.n_items * blockIdx.x / gridDim.x;
  const int64_t w1 = a.n_items * (blockIdx.x + 1) / gridDim.x;
  int cur_group = -1;
  const int64_t HG = a.H * G;

  for (int64_t w = w0; w < w1; ++w) {
    const int grp = (int)(w / n_pairs);
    const int64_t tp = w % n_pairs;
    const int u0 = grp * UG;
    const int nu = (int)min((int64_t)UG, a.B * a.H - u0);
    __syncthreads();  // previous item's readers are done with sc / constants
    if (grp != cur_group) {
      cur_group = grp;
      // Constants for every slot (unit, g) of the group.
      for (int s = threadIdx.x; s < slots; s += blockDim.x) sigma[s] = 0.f;
      __syncthreads();
      for (int idx = threadIdx.x; idx < nu * G * kPairs; idx += blockDim.x) {
        const int s = idx / kPairs, p = idx % kPairs;
        const int64_t u = u0 + s / G;
        const int64_t b = u / a.H, h = u % a.H;
        const int64_t hq = h * G + s % G;
        const __half* qv = a.q + (b * HG + hq) * kHeadDim;
        const float q1 = __half2float(qv[p]), q2 = __half2float(qv[p + 64]);
        const float s1 = a.k_scale[h * kHeadDim + p], s2 = a.k_scale[h * kHeadDim + p + 64];
        const float m = fmaxf(fmaxf(fabsf(s1 * q1), fabsf(s2 * q2)), fmaxf(fabsf(s1 * q2), fabsf(s2 * q1)));
        atomicMax(reinterpret_cast<int*>(sigma + s), __float_as_int(m));
      }
      __syncthreads();
      for (int idx = threadIdx.x; idx < nu * G * kPairs; idx += blockDim.x) {
        const int s = idx / kPairs, p = idx % kPairs;
        const int64_t u = u0 + s / G;
        const int64_t b = u / a.H, h = u % a.H;
        const int64_t hq = h * G + s % G;
        const __half* qv = a.q + (b * HG + hq) * kHeadDim;
        const float q1 = __half2float(qv[p]), q2 = __half2float(qv[p + 64]);
        const float s1 = a.k_scale[h * kHeadDim + p], s2 = a.k_scale[h * kHeadDim + p + 64];
        const float z1 = a.k_zero[h * kHeadDim + p], z2 = a.k_zero[h * kHeadDim + p + 64];
        // power-of-two normalizer so every fp16 constant is <= 1 in magnitude
        const float inv = ldexpf(1.f, -pow2_exponent(sigma[s]));
        KeyConst kc;
        kc.p12 = half2_bits(s1 * q1 * inv, s2 * q2 * inv);
        kc.q12 = half2_bits(s1 * q2 * inv, -s2 * q1 * inv);
        kc.ox = (z1 * q1 + z2 * q2) * inv;
        kc.oy = (z1 * q2 - z2 * q1) * inv;
        *key_const<BITS>(smem, s, p) = kc;
      }
      __syncthreads();
      __syncthreads();
      if (threadIdx.x < slots) sigma[threadIdx.x] = ldexpf(1.f, pow2_exponent(sigma[threadIdx.x]));
    }
    for (int idx = threadIdx.x; idx < slots * 64; idx += blockDim.x) sc[idx] = 0.f;

    // cos/sin for this lane's two tokens and the 16 pairs of chunk j.
    const int64_t tile0 = 2 * tp;
    float cs[2][16], sn[2][16];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int64_t t = (tile0 + r) * kTileTokens + lane;
#pragma unroll
      for (int m = 0; m < 16; ++m) rope_cos_sin(t, __ldg(a.inv_freq + 16 * j + m), cs[r][m], sn[r][m]);
    }
    __syncthreads();

    const bool has_b = tile0 + 1 < nt;
    const int64_t tbytes = kTileTokens * kHeadDim * BITS / 8;
    const int64_t slab_off = (int64_t)(j * 32 + lane) * (4 * BITS);
    CodeSlab<BITS> cur[2], nxt[2];
    auto load_unit = [&](int ui, CodeSlab<BITS>* dst) {
      const int64_t u = u0 + ui;
      const uint8_t* base = a.codes + (u * a.nt_cap + tile0) * tbytes + slab_off;
      dst[0].load(base);
      if (has_b) dst[1].load(base + tbytes);
      else { dst[1].w[0] = dst[1].w[1] = dst[1].w[2] = dst[1].w[3] = 0; }
    };
    load_unit(0, cur);
    for (int ui = 0; ui < nu; ++ui) {
      if (ui + 1 < nu) load_unit(ui + 1, nxt);
      float acc[G][2];
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const uint32_t l0 = *reinterpret_cast<const uint32_t*>(lut + PairLut<BITS>::addr(cur[0].w, m, lane4));
        const uint32_t l1 = *reinterpret_cast<const uint32_t*>(lut + PairLut<BITS>::addr(cur[1].w, m, lane4));
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const KeyConst kc = *key_const<BITS>(smem, ui * G + g, 16 * j + m);
          const uint16_t P1 = (uint16_t)lo16(kc.p12), P2 = (uint16_t)hi16(kc.p12);
          const uint16_t Q1 = (uint16_t)lo16(kc.q12), Q2 = (uint16_t)hi16(kc.q12);
          {
            const uint16_t L1 = (uint16_t)lo16(l0), L2 = (uint16_t)hi16(l0);
            const float X = fma_h(L1, P1, fma_h(L2, P2, kc.ox));
            const float Y = fma_h(L1, Q1, fma_h(L2, Q2, kc.oy));
            acc[g][0] = fmaf(cs[0][m], X, fmaf(sn[0][m], Y, acc[g][0]));
          }
          {
            const uint16_t L1 = (uint16_t)lo16(l1), L2 = (uint16_t)hi16(l1);
            const float X = fma_h(L1, P1, fma_h(L2, P2, kc.ox));
            const float Y = fma_h(L1, Q1, fma_h(L2, Q2, kc.oy));
            acc[g][1] = fmaf(cs[1][m], X, fmaf(sn[1][m], Y, acc[g][1]));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        atomicAdd(sc + (ui * G + g) * 64 + lane, acc[g][0]);
        atomicAdd(sc + (ui * G + g) * 64 + 32 + lane, acc[g][1]);
      }
      if (ui + 1 < nu) { cur[0] = nxt[0]; cur[1] = nxt[1]; }
    }
    __syncthreads();

    // Outliers: o * (cos * P + sin * Q) of the channel's half of the pair.
    for (int ui = 0; ui < nu; ++ui) {
      const int64_t u = u0 + ui;
      for (int r = 0; r < 2; ++r) {
        const int64_t tile = tile0 + r;
        if (tile >= nt) break;
        const int64_t e0 = a.out_ptr[u * a.nt_cap + tile], e1 = a.out_ptr[u * a.nt_cap + tile + 1];
        for (int64_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
          const uint32_t pos = a.out_pos[e];
          const int i = (int)((pos >> 7) & 31), d = (int)(pos & 127);
          const int p = d & 63, second = d >> 6;
          float c, s;
          rope_cos_sin(tile * kTileTokens + i, __ldg(a.inv_freq + p), c, s);
          const float o = __half2float(a.out_vals[e]);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const KeyConst kc = *key_const<BITS>(smem, ui * G + g, p);
            const __half2 pp = *reinterpret_cast<const __half2*>(&kc.p12);
            const __half2 qq = *reinterpret_cast<const __half2*>(&kc.q12);
            const float P = second ? __high2float(pp) : __low2float(pp);
            const float Q = second ? __high2float(qq) : __low2float(qq);
            atomicAdd(sc + (ui * G + g) * 64 + r * 32 + i, o * fmaf(c, P, s * Q));
          }
        }
      }
    }
    __syncthreads();

    // Sink token (position 0, no rotation): score = q . k_sink, fp32.
    if (tile0 == 0 && a.k_sink) {
      for (int s = j; s < nu * G; s += 4) {
        const int64_t u = u0 + s / G;
        const int64_t b = u / a.H, h = u % a.H;
        const int64_t hq = h * G + s % G;
        const __half* qv = a.q + (b * HG + hq) * kHeadDim;
        const __half* kv = a.k_sink + (b * a.H + h) * kHeadDim;
        float v = 0.f;
        for (int d = lane; d < kHeadDim; d += 32) v = fmaf(__half2float(qv[d]), __half2float(kv[d]), v);
        v = warp_sum(v);
        if (lane == 0) sc[s * 64] = v / sigma[s];
      }
      __syncthreads();
    }

    // Write out.
    for (int idx = threadIdx.x; idx < nu * G * 64; idx += blockDim.x) {
      const int s = idx / 64, tt = idx % 64;
      const int64_t t = tile0 * kTileTokens + tt;
      if (t >= a.T) continue;
      const int64_t u = u0 + s / G;
      const int64_t b = u / a.H, h = u % a.H;
      const int64_t hq = h * G + s % G;
      a.scores[(b * HG + hq) * a.T + t] = sc[idx] * sigma[s];
    }
  }
}

// ---------------------------------------------------------------------------
// Softmax along T of rows of scores * scale (two kernels over row chunks).
// ---------------------------------------------------------------------------
constexpr int kSoftmaxChunk = 4096;

__global__ void __launch_bounds__(256) softmax_partial_kernel(const float* __restrict__ x,
                                                               int64_t T, float scale,
                                                               float2* __restrict__ part) {
  __shared__ float rm[8], rl[8];
  const int64_t row = blockIdx.y, ch = blockIdx.x;
  const int64_t s = ch * kSoftmaxChunk, e = min(T, s + kSoftmaxChunk);
  const float* xr = x + row * T;
  float m = -INFINITY;
  for (int64_t t = s + threadIdx.x; t < e; t += blockDim.x) m = fmaxf(m, xr[t] * scale);
  m = warp_max(m);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) rm[w] = m;
  __syncthreads();
  m = rm[0];
  for (int i = 1; i < 8; ++i) m = fmaxf(m, rm[i]);
  float l = 0.f;
  for (int64_t t = s + threadIdx.x; t < e; t += blockDim.x) l += __expf(xr[t] * scale - m);
  l = warp_sum(l);
  if (lane == 0) rl[w] = l;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < 8; ++i) tot += rl[i];
    part[row * gridDim.x + ch] = make_float2(m, tot);
  }
}

__global__ void __launch_bounds__(256) softmax_write_kernel(const float* __restrict__ x,
                                                             int64_t T, float scale,
                                                             const float2* __restrict__ part,
                                                             float* __restrict__ p) {
  __shared__ float sm, sl;
  const int64_t row = blockIdx.y, ch = blockIdx.x;
  const int nch = gridDim.x;
  if (threadIdx.x < 32) {
    float m = -INFINITY;
    for (int i = threadIdx.x; i < nch; i += 32) m = fmaxf(m, part[row * nch + i].x);
    m = warp_max(m);
    float l = 0.f;
    for (int i = threadIdx.x; i < nch; i += 32) {
      const float2 pr = part[row * nch + i];
      l += pr.y * __expf(pr.x - m);
    }
    l = warp_sum(l);
    if (threadIdx.x == 0) { sm = m; sl = 1.f / l; }
  }
  __syncthreads();
  const float m = sm, il = sl;
  const int64_t s = ch * kSoftmaxChunk, e = min(T, s + kSoftmaxChunk);
  const float* xr = x + row * T;
  float* pr = p + row * T;
  for (int64_t t = s + threadIdx.x; t < e; t += blockDim.x) pr[t] = __expf(xr[t] * scale - m) * il;
}

// ---------------------------------------------------------------------------
// Value kernel. One CTA = 4 warps (chunks of 32 channels) x 32 token lanes;
// a work item is (unit, split of tiles); each thread accumulates its 32
// channels over one token per tile for the G query heads of the unit.
// ---------------------------------------------------------------------------
struct ValueArgs {
  const uint8_t* codes;
  const __half* out_vals;
  const uint16_t* out_pos;
  const int32_t* out_ptr;
  const float* v_scale;  // [B, ld]
  const float* v_zero;
  int64_t ld;
  const __half* v_sink;  // [B, H*128] or null
  const float* cb;
  const float* probs;    // [B, H*G, T]
  int64_t B, H, G, T, nt_cap;
  int n_splits;
  float* partial;        // [n_splits, B*H*G, 129]: 128 channels + zero term
};

constexpr int kValThreads = 128;

template <int BITS, int G>
__global__ void __launch_bounds__(kValThreads) value_kernel(ValueArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* lut = smem;
  float* red = reinterpret_cast<float*>(smem + PairLut<BITS>::kBytes);  // [4 warps][32][33]
  __shared__ float s_e[G];         // per-slot power-of-two weight scale
  __shared__ float s_acc[G][129];  // outliers + zero term + sink (fp32, unscaled)
  const int j = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lane4 = (uint32_t)lane << 2;
  PairLut<BITS>::build(lut, a.cb);

  const int64_t nt = (a.T + kTileTokens - 1) / kTileTokens;
  const int64_t U = a.B * a.H;
  const int64_t item = blockIdx.x;  // over U * n_splits
  const int64_t u = item / a.n_splits;
  const int split = (int)(item % a.n_splits);
  const int64_t tpb = (nt + a.n_splits - 1) / a.n_splits;
  const int64_t ta = split * tpb, tb = min(nt, ta + tpb);
  const int64_t b = u / a.H, h = u % a.H;
  const int64_t HG = a.H * G;
  const bool sink = a.v_sink != nullptr;
  const float* vs = a.v_scale + b * a.ld;
  const float* vz = a.v_zero + b * a.ld;

  // Pass 1: largest weight p_t * s_t per slot in this split -> fp16 scale.
  for (int idx = threadIdx.x; idx < G * 129; idx += blockDim.x) (&s_acc[0][0])[idx] = 0.f;
  __syncthreads();
  {
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mx[g] = 0.f;
    for (int64_t t = ta * kTileTokens + threadIdx.x; t < min(a.T, tb * kTileTokens); t += blockDim.x) {
      if (sink && t == 0) continue;
      const float s = vs[t];
#pragma unroll
      for (int g = 0; g < G; ++g) mx[g] = fmaxf(mx[g], a.probs[(b * HG + h * G + g) * a.T + t] * s);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float m = warp_max(mx[g]);
      if (lane == 0) atomicMax(reinterpret_cast<int*>(&s_acc[g][128]), __float_as_int(m));
    }
  }
  __syncthreads();
  if (threadIdx.x < G)  // largest weight <= 2^14 in fp16
    s_e[threadIdx.x] = ldexpf(1.f, 14 - pow2_exponent(s_acc[threadIdx.x][128]));
  __syncthreads();
  if (threadIdx.x < G) s_acc[threadIdx.x][128] = 0.f;
  __syncthreads();

  float acc[G][32];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < 32; ++c) acc[g][c] = 0.f;
  float zsum[G];
#pragma unroll
  for (int g = 0; g < G; ++g) zsum[g] = 0.f;
  float e_scale[G];
#pragma unroll
  for (int g = 0; g < G; ++g) e_scale[g] = s_e[g];

  const int64_t tbytes = kTileTokens * kHeadDim * BITS / 8;
  const int64_t slab_off = (int64_t)(j * 32 + lane) * (4 * BITS);
  const uint8_t* ubase = a.codes + u * a.nt_cap * tbytes + slab_off;
  CodeSlab<BITS> cur;
  if (ta < tb) cur.load(ubase + ta * tbytes);
  for (int64_t tile = ta; tile < tb; ++tile) {
    CodeSlab<BITS> nxt;
    if (tile + 1 < tb) nxt.load(ubase + (tile + 1) * tbytes);
    const int64_t t = tile * kTileTokens + lane;
    uint16_t w16[G];
    const bool live = t < a.T && !(sink && t == 0);
    const float s_t = live ? vs[t] : 0.f;
    const float z_t = live ? vz[t] : 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float p = live ? a.probs[(b * HG + h * G + g) * a.T + t] : 0.f;
      const __half hw = __float2half_rn(p * s_t * e_scale[g]);
      w16[g] = *reinterpret_cast<const uint16_t*>(&hw);
      if (j == 0) zsum[g] = fmaf(p, z_t, zsum[g]);
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const uint32_t l = *reinterpret_cast<const uint32_t*>(lut + PairLut<BITS>::addr(cur.w, m, lane4));
#pragma unroll
      for (int g = 0; g < G; ++g) {
        acc[g][2 * m] = fma_h((uint16_t)lo16(l), w16[g], acc[g][2 * m]);
        acc[g][2 * m + 1] = fma_h((uint16_t)hi16(l), w16[g], acc[g][2 * m + 1]);
      }
    }
    if (tile + 1 < tb) cur = nxt;
  }
  // Outliers of this split: p_t * s_t * o into channel d.
  for (int64_t tile = ta; tile < tb; ++tile) {
    const int64_t e0 = a.out_ptr[u * a.nt_cap + tile], e1 = a.out_ptr[u * a.nt_cap + tile + 1];
    for (int64_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
      const uint32_t pos = a.out_pos[e];
      const int64_t t = tile * kTileTokens + (pos >> 7);
      const int d = (int)(pos & 127);
      if (t >= a.T || (sink && t == 0)) continue;
      const float os = __half2float(a.out_vals[e]) * vs[t];
#pragma unroll
      for (int g = 0; g < G; ++g)
        atomicAdd(&s_acc[g][d], a.probs[(b * HG + h * G + g) * a.T + t] * os);
    }
  }
  // Sink (token 0 in the first split).
  if (sink && ta == 0 && a.T > 0) {
    for (int idx = threadIdx.x; idx < G * kHeadDim; idx += blockDim.x) {
      const int g = idx / kHeadDim, d = idx % kHeadDim;
      const float p0 = a.probs[(b * HG + h * G + g) * a.T];
      atomicAdd(&s_acc[g][d], p0 * __half2float(a.v_sink[(b * a.H + h) * kHeadDim + d]));
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float z = warp_sum(zsum[g]);
    if (j == 0 && lane == 0) atomicAdd(&s_acc[g][128], z);
  }
  // Reduce the 32 token lanes of each warp (channels 32j..32j+31).
  for (int g = 0; g < G; ++g) {
    __syncthreads();
    float* r = red + j * 32 * 33;
#pragma unroll
    for (int c = 0; c < 32; ++c) r[lane * 33 + c] = acc[g][c];
    __syncwarp();
    float sum = 0.f;
    for (int l2 = 0; l2 < 32; ++l2) sum += r[l2 * 33 + lane];
    const int d = 32 * j + lane;
    const float inv = 1.f / e_scale[g];
    float* dst = a.partial + ((int64_t)split * (U * G) + u * G + g) * 129;
    __syncthreads();
    dst[d] = sum * inv + s_acc[g][d];
    if (threadIdx.x == 0) dst[128] = s_acc[g][128];
  }
}

// out[slot, d] = sum over splits (partial[d] + zero term), as fp16.
__global__ void value_combine_kernel(const float* __restrict__ partial, int n_splits,
                                     int64_t n_slots, __half* __restrict__ out) {
  const int64_t slot = blockIdx.x;
  const int d = threadIdx.x;  // 128 threads
  float v = 0.f, z = 0.f;
  for (int s = 0; s < n_splits; ++s) {
    const float* p = partial + ((int64_t)s * n_slots + slot) * 129;
    v += p[d];
    z += p[128];
  }
  out[slot * kHeadDim + d] = __float2half_rn(v + z);
}

inline int value_splits(int64_t U, int64_t nt) {
  // enough CTAs to fill the GPU (148 SMs x ~4 resident) but >= 8 tiles each
  int64_t s = (148 * 4 + U - 1) / U;
  const int64_t max_s = (nt + 7) / 8;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  return (int)s;
}

}  // namespace kvq

namespace kvq {

template <int BITS, int G>
static int launch_key(const KeyArgs& a0, cudaStream_t st) {
  KeyArgs a = a0;
  const int64_t U = a.B * a.H;
  const int UG = (int)(U < (int64_t)(kMaxSlots / G) ? U : (int64_t)(kMaxSlots / G));
  a.units_per_group = UG;
  a.n_groups = (int)((U + UG - 1) / UG);
  const int64_t nt = (a.T + kTileTokens - 1) / kTileTokens;
  const int64_t n_pairs = (nt + 1) / 2;
  a.n_items = n_pairs * a.n_groups;
  const int smem = key_smem_bytes<BITS>();
  cudaFuncSetAttribute(key_scores_kernel<BITS, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, key_scores_kernel<BITS, G>, kKeyThreads, smem);
  if (per_sm < 1) per_sm = 1;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t grid = (int64_t)sms * per_sm;
  if (grid > a.n_items) grid = a.n_items;
  if (grid < 1) grid = 1;
  key_scores_kernel<BITS, G><<<(unsigned)grid, kKeyThreads, smem, st>>>(a);
  return check_launch("key_scores");
}

template <int BITS, int G>
static int launch_value(const ValueArgs& a0, cudaStream_t st) {
  ValueArgs a = a0;
  const int smem = PairLut<BITS>::kBytes + 4 * 32 * 33 * 4;
  cudaFuncSetAttribute(value_kernel<BITS, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int64_t U = a.B * a.H;
  value_kernel<BITS, G><<<(unsigned)(U * a.n_splits), kValThreads, smem, st>>>(a);
  return check_launch("value_output");
}

template <int G>
static int dispatch_key_bits(int bits, const KeyArgs& a, cudaStream_t st) {
  switch (bits) {
    case 2: return launch_key<2, G>(a, st);
    case 3: return launch_key<3, G>(a, st);
    case 4: return launch_key<4, G>(a, st);
  }
  set_error("key_scores: bits must be 2, 3 or 4 (got %d)", bits);
  return KVQ_ERR_UNSUPPORTED;
}

template <int G>
static int dispatch_value_bits(int bits, const ValueArgs& a, cudaStream_t st) {
  switch (bits) {
    case 2: return launch_value<2, G>(a, st);
    case 3: return launch_value<3, G>(a, st);
    case 4: return launch_value<4, G>(a, st);
  }
  set_error("value_output: bits must be 2, 3 or 4 (got %d)", bits);
  return KVQ_ERR_UNSUPPORTED;
}

static int check_decode_shape(const char* what, int64_t B, int64_t H, int64_t G, int64_t T,
                              int64_t nt_cap) {
  if (B < 1 || H < 1 || T < 1 || nt_cap * kTileTokens < T) {
    set_error("%s: invalid shape B=%lld H=%lld T=%lld nt_cap=%lld", what, (long long)B,
              (long long)H, (long long)T, (long long)nt_cap);
    return KVQ_ERR_INVALID;
  }
  if (!(G == 1 || G == 2 || G == 4 || G == 8)) {
    set_error("%s: group (query heads per KV head) must be 1, 2, 4 or 8 (got %lld)", what,
              (long long)G);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (T >= (1LL << 30)) {
    set_error("%s: T too large", what);
    return KVQ_ERR_INVALID;
  }
  return KVQ_OK;
}

}  // namespace kvq

extern "C" int kvq_key_scores(const uint8_t* codes, const void* out_vals, const uint16_t* out_pos,
                              const int32_t* out_ptr, const float* k_scale, const float* k_zero,
                              const void* k_sink, const float* codebook, int bits, const void* q,
                              const float* inv_freq, int64_t B, int64_t n_heads, int64_t group,
                              int64_t T, int64_t nt_cap, float* scores, void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_decode_shape("key_scores", B, n_heads, group, T, nt_cap);
  if (rc) return rc;
  KeyArgs a{};
  a.codes = codes; a.out_vals = (const __half*)out_vals; a.out_pos = out_pos;
  a.out_ptr = out_ptr; a.k_scale = k_scale; a.k_zero = k_zero; a.k_sink = (const __half*)k_sink;
  a.cb = codebook; a.q = (const __half*)q; a.inv_freq = inv_freq; a.B = B; a.H = n_heads;
  a.G = group; a.T = T; a.nt_cap = nt_cap; a.scores = scores;
  cudaStream_t st = as_stream(stream);
  switch (group) {
    case 1: return dispatch_key_bits<1>(bits, a, st);
    case 2: return dispatch_key_bits<2>(bits, a, st);
    case 4: return dispatch_key_bits<4>(bits, a, st);
    case 8: return dispatch_key_bits<8>(bits, a, st);
  }
  return KVQ_ERR_UNSUPPORTED;
}

extern "C" size_t kvq_softmax_workspace(int64_t rows, int64_t T) {
  const int64_t nch = (T + kvq::kSoftmaxChunk - 1) / kvq::kSoftmaxChunk;
  return kvq::align256((size_t)(rows > 0 ? rows : 0) * (nch > 0 ? nch : 0) * sizeof(float2));
}

namespace kvq {
static int softmax_impl(const float* scores, int64_t rows, int64_t T, float scale, float* probs,
                        void* workspace, size_t workspace_bytes, cudaStream_t st) {
  if (rows < 0 || T < 1) {
    set_error("softmax: invalid shape rows=%lld T=%lld", (long long)rows, (long long)T);
    return KVQ_ERR_INVALID;
  }
  if (rows == 0) return KVQ_OK;
  const int64_t nch = (T + kSoftmaxChunk - 1) / kSoftmaxChunk;
  if (nch > 65535 || rows > 65535) {
    set_error("softmax: too large (rows=%lld, T=%lld)", (long long)rows, (long long)T);
    return KVQ_ERR_INVALID;
  }
  if (!workspace || workspace_bytes < (size_t)rows * nch * sizeof(float2)) {
    set_error("softmax: workspace too small");
    return KVQ_ERR_INVALID;
  }
  float2* part = reinterpret_cast<float2*>(workspace);
  dim3 g((unsigned)nch, (unsigned)rows);
  softmax_partial_kernel<<<g, 256, 0, st>>>(scores, T, scale, part);
  softmax_write_kernel<<<g, 256, 0, st>>>(scores, T, scale, part, probs);
  return check_launch("softmax");
}

static int value_impl(const uint8_t* codes, const void* out_vals, const uint16_t* out_pos,
                      const int32_t* out_ptr, const float* v_scale, const float* v_zero,
                      int64_t ld_stats, const void* v_sink, const float* codebook, int bits,
                      const float* probs, int64_t B, int64_t H, int64_t G, int64_t T,
                      int64_t nt_cap, void* out, void* workspace, size_t workspace_bytes,
                      cudaStream_t st) {
  int rc = check_decode_shape("value_output", B, H, G, T, nt_cap);
  if (rc) return rc;
  if (ld_stats < T) {
    set_error("value_output: ld_stats=%lld < T=%lld", (long long)ld_stats, (long long)T);
    return KVQ_ERR_INVALID;
  }
  const int64_t U = B * H;
  const int64_t nt = (T + kTileTokens - 1) / kTileTokens;
  const int n_splits = value_splits(U, nt);
  const size_t need = (size_t)n_splits * U * G * 129 * sizeof(float);
  if (!workspace || workspace_bytes < need) {
    set_error("value_output: workspace too small (%zu < %zu)", workspace_bytes, need);
    return KVQ_ERR_INVALID;
  }
  ValueArgs a{};
  a.codes = codes; a.out_vals = (const __half*)out_vals; a.out_pos = out_pos;
  a.out_ptr = out_ptr; a.v_scale = v_scale; a.v_zero = v_zero; a.ld = ld_stats;
  a.v_sink = (const __half*)v_sink; a.cb = codebook; a.probs = probs; a.B = B; a.H = H;
  a.G = G; a.T = T; a.nt_cap = nt_cap; a.n_splits = n_splits;
  a.partial = reinterpret_cast<float*>(workspace);
  switch (G) {
    case 1: rc = dispatch_value_bits<1>(bits, a, st); break;
    case 2: rc = dispatch_value_bits<2>(bits, a, st); break;
    case 4: rc = dispatch_value_bits<4>(bits, a, st); break;
    case 8: rc = dispatch_value_bits<8>(bits, a, st); break;
    default: rc = KVQ_ERR_UNSUPPORTED;
  }
  if (rc) return rc;
  value_combine_kernel<<<(unsigned)(U * G), kHeadDim, 0, st>>>(a.partial, n_splits, U * G,
                                                                 (__half*)out);
  return check_launch("value_output");
}

inline size_t value_ws(int64_t B, int64_t H, int64_t G, int64_t T) {
  const int64_t U = B * H;
  const int64_t nt = (T + kTileTokens - 1) / kTileTokens;
  return align256((size_t)value_splits(U, nt) * U * G * 129 * sizeof(float));
}
}  // namespace kvq

extern "C" int kvq_softmax(const float* scores, int64_t rows, int64_t T, float scale,
                           float* probs, void* workspace, size_t workspace_bytes, void* stream) {
  kvq::clear_error();
  return kvq::softmax_impl(scores, rows, T, scale, probs, workspace, workspace_bytes,
                           kvq::as_stream(stream));
}

extern "C" size_t kvq_value_output_workspace(int64_t B, int64_t n_heads, int64_t group,
                                             int64_t T) {
  return kvq::value_ws(B, n_heads, group, T);
}

extern "C" int kvq_value_output(const uint8_t* codes, const void* out_vals,
                                const uint16_t* out_pos, const int32_t* out_ptr,
                                const float* v_scale, const float* v_zero, int64_t ld_stats,
                                const void* v_sink, const float* codebook, int bits,
                                const float* probs, int64_t B, int64_t n_heads, int64_t group,
                                int64_t T, int64_t nt_cap, void* out, void* workspace,
                                size_t workspace_bytes, void* stream) {
  kvq::clear_error();
  return kvq::value_impl(codes, out_vals, out_pos, out_ptr, v_scale, v_zero, ld_stats, v_sink,
                         codebook, bits, probs, B, n_heads, group, T, nt_cap, out, workspace,
                         workspace_bytes, kvq::as_stream(stream));
}

namespace kvq {
// Workspace of decode_attention: [scores][probs][softmax partials][value partials].
struct DecodeWs {
  size_t scores, probs, soft, value, total;
};
inline DecodeWs decode_ws(int64_t B, int64_t H, int64_t G, int64_t T) {
  DecodeWs w;
  const int64_t rows = B * H * G;
  w.scores = align256((size_t)rows * T * sizeof(float));
  w.probs = w.scores;
  w.soft = kvq_softmax_workspace(rows, T);
  w.value = value_ws(B, H, G, T);
  w.total = w.scores + w.probs + w.soft + w.value;
  return w;
}
}  // namespace kvq

extern "C" size_t kvq_decode_attention_workspace(int64_t B, int64_t n_heads, int64_t group,
                                                 int64_t T) {
  return kvq::decode_ws(B, n_heads, group, T).total;
}

extern "C" int kvq_decode_attention(
    const uint8_t* k_codes, const void* k_out_vals, const uint16_t* k_out_pos,
    const int32_t* k_out_ptr, const float* k_scale, const float* k_zero, const void* k_sink,
    const float* k_codebook, const uint8_t* v_codes, const void* v_out_vals,
    const uint16_t* v_out_pos, const int32_t* v_out_ptr, const float* v_scale,
    const float* v_zero, int64_t ld_stats, const void* v_sink, const float* v_codebook, int bits,
    const void* q, const float* inv_freq, int64_t B, int64_t n_heads, int64_t group, int64_t T,
    int64_t nt_cap, void* out, float* scores_out, float* probs_out, void* workspace,
    size_t workspace_bytes, void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_decode_shape("decode_attention", B, n_heads, group, T, nt_cap);
  if (rc) return rc;
  const DecodeWs w = decode_ws(B, n_heads, group, T);
  if (!workspace || workspace_bytes < w.total) {
    set_error("decode_attention: workspace too small (%zu < %zu)", workspace_bytes, w.total);
    return KVQ_ERR_INVALID;
  }
  char* ws = reinterpret_cast<char*>(workspace);
  float* scores = scores_out ? scores_out : reinterpret_cast<float*>(ws);
  float* probs = probs_out ? probs_out : reinterpret_cast<float*>(ws + w.scores);
  void* soft = ws + w.scores + w.probs;
  void* val = ws + w.scores + w.probs + w.soft;
  rc = kvq_key_scores(k_codes, k_out_vals, k_out_pos, k_out_ptr, k_scale, k_zero, k_sink,
                      k_codebook, bits, q, inv_freq, B, n_heads, group, T, nt_cap, scores, stream);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  rc = softmax_impl(scores, B * n_heads * group, T, 0.08838834764831845f /* 1/sqrt(128) */,
                    probs, soft, w.soft, st);
  if (rc) return rc;
  return value_impl(v_codes, v_out_vals, v_out_pos, v_out_ptr, v_scale, v_zero, ld_stats, v_sink,
                    v_codebook, bits, probs, B, n_heads, group, T, nt_cap, out, val, w.value, st);
}
