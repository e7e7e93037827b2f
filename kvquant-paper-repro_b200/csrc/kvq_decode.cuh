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
// fp16 x fp16 + fp32 FMA; outliers are added from the tile-CSR.
//
// Value kernel: out[b,hq,:] = sum_t p_t * (s_t * (cb[code] + o) + z_t) with the
// per-token scale s_t / zero z_t over all channels (kv_quantizer.py:103-117).
//
// Both kernels stream their codes (and the per-token data and outlier entries
// they need) through a per-thread cp.async ring in shared memory: every thread
// copies exactly the bytes it will read itself, so the only synchronisation is
// cp.async.wait_group, and the copies of several units / tiles stay in flight.
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

// ---------------------------------------------------------------------------
// cp.async helpers (sizes 4/8/16; src_bytes < size zero-fills the rest and
// src_bytes == 0 reads nothing).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t n) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint32_t n) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t n) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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

// One thread's code slab (4*BITS bytes), copied into / read from shared memory.
template <int BITS>
struct CodeSlab {
  uint32_t w[4];
  // Asynchronous copy of the slab at src into the 16-byte smem slot dst.
  __device__ static __forceinline__ void copy(uint32_t dst, const uint8_t* src, bool valid) {
    if (BITS == 4) {
      cp_async16(dst, src, valid ? 16u : 0u);
    } else if (BITS == 2) {
      cp_async8(dst, src, valid ? 8u : 0u);
    } else {
      cp_async4(dst, src, valid ? 4u : 0u);
      cp_async4(dst + 4, src + 4, valid ? 4u : 0u);
      cp_async4(dst + 8, src + 8, valid ? 4u : 0u);
    }
  }
  __device__ __forceinline__ void read(const uint8_t* slot) {
    if (BITS == 4) {
      const uint4 v = *reinterpret_cast<const uint4*>(slot);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if (BITS == 2) {
      const uint2 v = *reinterpret_cast<const uint2*>(slot);
      w[0] = v.x; w[1] = v.y; w[2] = 0; w[3] = 0;
    } else {
      const uint32_t* q = reinterpret_cast<const uint32_t*>(slot);
      w[0] = q[0]; w[1] = q[1]; w[2] = q[2]; w[3] = 0;
    }
  }
};

__device__ __forceinline__ float entry_value(uint32_t ent) {
  return __half2float(__ushort_as_half((unsigned short)(ent >> 16)));
}

// ===========================================================================
// Key kernel
// ===========================================================================
// Per-(slot, pair) key constants, 16 bytes: fp16 {P1, P2} {Q1, Q2}, fp32 OX, OY
// (all divided by the slot's power-of-two sigma).
struct KeyConst {
  uint32_t p12, q12;
  float ox, oy;
};

struct KeyArgs {
  const uint8_t* codes;
  const uint32_t* out_ent;
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
  int64_t n_items;       // tile quads * groups
};

// CTA = 8 warps: warp w handles chunk j = w & 3 (16 RoPE pairs) of tiles
// 2*(w >> 2) and 2*(w >> 2) + 1 of a 4-tile (128-token) work item; every
// thread keeps cos/sin of its two tokens x 16 pairs in registers.
constexpr int kKeyThreads = 256;
constexpr int kKeyTiles = 4;                     // tiles per work item
constexpr int kKeyTokens = kKeyTiles * kTileTokens;
constexpr int kMaxSlots = 32;                    // query heads per group
constexpr int kKeyStages = 3;                    // units in flight per thread

// Shared-memory layout of the key kernel: pair LUT, per-slot constants, score
// accumulators, per-slot normalizers, per-unit outlier row pointers and the
// cp.async ring (per stage: 2 x 16-byte slab slots + one outlier entry per
// thread). For 4-bit codes the constants live in bytes 128..255 of the LUT's
// 256-byte rows (32 slots x 64 pairs x 16 B).
template <int BITS>
struct KeySmem {
  static constexpr int kLut = PairLut<BITS>::kBytes;
  static constexpr int kConst = BITS == 4 ? 0 : kLut;
  static constexpr int kSc = BITS == 4 ? kLut : kConst + kMaxSlots * kPairs * 16;
  static constexpr int kSigma = kSc + kMaxSlots * kKeyTokens * 4;
  static constexpr int kPtr = kSigma + kMaxSlots * 4;  // [slots][kKeyTiles + 1] int32
  static constexpr int kRing = kPtr + kMaxSlots * (kKeyTiles + 1) * 4;
  static constexpr int kRingSlab = kKeyThreads * 32;    // per stage: [2][thread][16 B]
  static constexpr int kRingEnt = kKeyThreads * 4;      // per stage: [thread] uint32
  static constexpr int kBytes = kRing + kKeyStages * (kRingSlab + kRingEnt);
};

template <int BITS>
__host__ __device__ constexpr int key_smem_bytes() { return KeySmem<BITS>::kBytes; }

template <int BITS>
__device__ __forceinline__ KeyConst* key_const(uint8_t* smem, int slot, int p) {
  const int idx = slot * kPairs + p;  // < 2048 16-byte cells
  if (BITS == 4)
    return reinterpret_cast<KeyConst*>(smem + ((idx >> 3) << 8) + 128 + ((idx & 7) << 4));
  return reinterpret_cast<KeyConst*>(smem + KeySmem<BITS>::kConst) + idx;
}

#ifndef KVQ_KEY_MIN_BLOCKS
#define KVQ_KEY_MIN_BLOCKS 2  // resident CTAs per SM the register budget targets
#endif

template <int BITS, int G>
__global__ void __launch_bounds__(kKeyThreads, KVQ_KEY_MIN_BLOCKS) key_scores_kernel(KeyArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  using L = KeySmem<BITS>;
  uint8_t* lut = smem;
  float* sc = reinterpret_cast<float*>(smem + L::kSc);        // [slots][128 tokens]
  float* sigma = reinterpret_cast<float*>(smem + L::kSigma);  // [slots]
  int32_t* uptr = reinterpret_cast<int32_t*>(smem + L::kPtr);  // [units][kKeyTiles + 1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = warp & 3, half = warp >> 2;
  const uint32_t lane4 = (uint32_t)lane << 2;
  PairLut<BITS>::build(lut, a.cb);
  // This thread's ring slots.
  uint8_t* ring_slab = smem + L::kRing + threadIdx.x * 16;  // + kKeyThreads*16 for slab 1
  uint32_t* ring_ent = reinterpret_cast<uint32_t*>(smem + L::kRing + kKeyStages * L::kRingSlab) +
                       threadIdx.x;

  const int64_t nt = (a.T + kTileTokens - 1) / kTileTokens;
  const int64_t n_quads = (nt + kKeyTiles - 1) / kKeyTiles;
  const int UG = a.units_per_group;
  const int slots = UG * G;
  // Static contiguous split of the (group-major) work list.
  const int64_t w0 = a.n_items * blockIdx.x / gridDim.x;
  const int64_t w1 = a.n_items * (blockIdx.x + 1) / gridDim.x;
  int cur_group = -1;
  const int64_t HG = a.H * G;
  const int64_t tbytes = kTileTokens * kHeadDim * BITS / 8;
  const int64_t slab_off = (int64_t)(j * 32 + lane) * (4 * BITS);

  for (int64_t w = w0; w < w1; ++w) {
    const int grp = (int)(w / n_quads);
    const int64_t tq = w % n_quads;
    const int u0 = grp * UG;
    const int nu = (int)min((int64_t)UG, a.B * a.H - u0);
    __syncthreads();  // previous item's readers are done with sc / tables
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
      if (threadIdx.x < slots) sigma[threadIdx.x] = ldexpf(1.f, pow2_exponent(sigma[threadIdx.x]));
    }
    for (int idx = threadIdx.x; idx < slots * kKeyTokens; idx += blockDim.x) sc[idx] = 0.f;
    const int64_t tile0 = kKeyTiles * tq;
    const int ntiles = (int)min((int64_t)kKeyTiles, nt - tile0);
    // Outlier row pointers of every unit over the item's tiles.
    for (int idx = threadIdx.x; idx < nu * (kKeyTiles + 1); idx += blockDim.x) {
      const int ui = idx / (kKeyTiles + 1), k = idx % (kKeyTiles + 1);
      uptr[idx] = __ldg(a.out_ptr + (u0 + ui) * a.nt_cap + tile0 + min(k, ntiles));
    }
    __syncthreads();  // uptr is read by the copy issue below

    const int64_t my_tile = tile0 + 2 * half;  // this thread's tiles: my_tile, my_tile + 1
    const bool has0 = my_tile < nt, has1 = my_tile + 1 < nt;

    // Issue the copies of unit ui into ring stage ui % kKeyStages (always one
    // commit per call so group counting stays uniform).
    auto issue = [&](int ui) {
      if (ui < nu) {
        const int st = ui % kKeyStages;
        const int64_t u = u0 + ui;
        const uint8_t* base = a.codes + (u * a.nt_cap + (has0 ? my_tile : tile0)) * tbytes + slab_off;
        const uint32_t dst = smem_u32(ring_slab + st * L::kRingSlab);
        CodeSlab<BITS>::copy(dst, base, has0);
        CodeSlab<BITS>::copy(dst + kKeyThreads * 16, has1 ? base + tbytes : base, has1);
        const int32_t e0 = uptr[ui * (kKeyTiles + 1)], e1 = uptr[ui * (kKeyTiles + 1) + ntiles];
        const int32_t e = e0 + (int32_t)threadIdx.x;
        cp_async4(smem_u32(ring_ent + st * kKeyThreads), a.out_ent + (e < e1 ? e : 0),
                  e < e1 ? 4u : 0u);
      }
      cp_async_commit();
    };

    // cos/sin for this thread's two tokens and the 16 pairs of chunk j
    // (computed while the first units' copies are in flight).
    for (int ui = 0; ui < kKeyStages - 1; ++ui) issue(ui);
    float cs[2][16], sn[2][16];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int64_t t = (my_tile + r) * kTileTokens + lane;
#pragma unroll
      for (int m = 0; m < 16; ++m) rope_cos_sin(t, __ldg(a.inv_freq + 16 * j + m), cs[r][m], sn[r][m]);
    }

    for (int ui = 0; ui < nu; ++ui) {
      issue(ui + kKeyStages - 1);
      cp_async_wait<kKeyStages - 1>();
      const int st = ui % kKeyStages;
      CodeSlab<BITS> s0, s1;
      s0.read(ring_slab + st * L::kRingSlab);
      s1.read(ring_slab + st * L::kRingSlab + kKeyThreads * 16);
      const int32_t e0 = uptr[ui * (kKeyTiles + 1)], e1 = uptr[ui * (kKeyTiles + 1) + ntiles];
      const int32_t e_first = e0 + (int32_t)threadIdx.x;
      uint32_t ent = ring_ent[st * kKeyThreads];

      float acc[G][2];
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const uint32_t l0 = *reinterpret_cast<const uint32_t*>(lut + PairLut<BITS>::addr(s0.w, m, lane4));
        const uint32_t l1 = *reinterpret_cast<const uint32_t*>(lut + PairLut<BITS>::addr(s1.w, m, lane4));
        uint16_t A1, A2, B1, B2;
        unpack16(l0, A1, A2);
        unpack16(l1, B1, B2);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const KeyConst kc = *key_const<BITS>(smem, ui * G + g, 16 * j + m);
          uint16_t P1, P2, Q1, Q2;
          unpack16(kc.p12, P1, P2);
          unpack16(kc.q12, Q1, Q2);
          {
            const float X = fma_h(A1, P1, fma_h(A2, P2, kc.ox));
            const float Y = fma_h(A1, Q1, fma_h(A2, Q2, kc.oy));
            acc[g][0] = fmaf(cs[0][m], X, fmaf(sn[0][m], Y, acc[g][0]));
          }
          {
            const float X = fma_h(B1, P1, fma_h(B2, P2, kc.ox));
            const float Y = fma_h(B1, Q1, fma_h(B2, Q2, kc.oy));
            acc[g][1] = fmaf(cs[1][m], X, fmaf(sn[1][m], Y, acc[g][1]));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        atomicAdd(sc + (ui * G + g) * kKeyTokens + (2 * half) * 32 + lane, acc[g][0]);
        atomicAdd(sc + (ui * G + g) * kKeyTokens + (2 * half + 1) * 32 + lane, acc[g][1]);
      }
      // Outliers: o * (cos * P + sin * Q) of the channel's half of the pair,
      // with the exact-angle cos/sin (an fp16 table would cost ~1e-3 on
      // outlier-heavy scores).
      if (e_first < e1) {
        int32_t bnd[kKeyTiles - 1];
#pragma unroll
        for (int k = 1; k < kKeyTiles; ++k) bnd[k - 1] = uptr[ui * (kKeyTiles + 1) + k];
        for (int32_t e = e_first; e < e1; e += kKeyThreads) {
          if (e != e_first) ent = __ldg(a.out_ent + e);
          int k = 0;
#pragma unroll
          for (int q = 0; q < kKeyTiles - 1; ++q) k += e >= bnd[q] ? 1 : 0;
          const int tok = k * kTileTokens + (int)((ent >> 7) & 31);
          const int ch = (int)(ent & 127);
          const int p = ch & 63, second = ch >> 6;
          const float oval = entry_value(ent);
          float c, sv;
          rope_cos_sin(tile0 * kTileTokens + tok, __ldg(a.inv_freq + p), c, sv);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const KeyConst kc = *key_const<BITS>(smem, ui * G + g, p);
            const __half2 pp = *reinterpret_cast<const __half2*>(&kc.p12);
            const __half2 qq = *reinterpret_cast<const __half2*>(&kc.q12);
            const float P = second ? __high2float(pp) : __low2float(pp);
            const float Q = second ? __high2float(qq) : __low2float(qq);
            atomicAdd(sc + (ui * G + g) * kKeyTokens + tok, oval * fmaf(c, P, sv * Q));
          }
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();

    // Sink token (position 0, no rotation): score = q . k_sink, fp32.
    if (tile0 == 0 && a.k_sink) {
      for (int s = warp; s < nu * G; s += kKeyThreads / 32) {
        const int64_t u = u0 + s / G;
        const int64_t b = u / a.H, h = u % a.H;
        const int64_t hq = h * G + s % G;
        const __half* qv = a.q + (b * HG + hq) * kHeadDim;
        const __half* kv = a.k_sink + (b * a.H + h) * kHeadDim;
        float v = 0.f;
        for (int dd = lane; dd < kHeadDim; dd += 32) v = fmaf(__half2float(qv[dd]), __half2float(kv[dd]), v);
        v = warp_sum(v);
        if (lane == 0) sc[s * kKeyTokens] = v / sigma[s];
      }
      __syncthreads();
    }

    // Write out.
    for (int idx = threadIdx.x; idx < nu * G * kKeyTokens; idx += blockDim.x) {
      const int s = idx / kKeyTokens, tt = idx % kKeyTokens;
      const int64_t t = tile0 * kTileTokens + tt;
      if (t >= a.T) continue;
      const int64_t u = u0 + s / G;
      const int64_t b = u / a.H, h = u % a.H;
      const int64_t hq = h * G + s % G;
      a.scores[(b * HG + hq) * a.T + t] = sc[idx] * sigma[s];
    }
  }
}

// ===========================================================================
// Softmax along T of rows of scores * scale (two kernels over row chunks).
// ===========================================================================
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

// ===========================================================================
// Value kernel. One CTA = 8 warps: warp w handles chunk j = w & 3 (32
// channels) of the tiles of parity w >> 2; a work item is (unit, split of
// tiles); each thread accumulates its 32 channels over one token per tile for
// the G query heads of the unit.
// ===========================================================================
struct ValueArgs {
  const uint8_t* codes;
  const uint32_t* out_ent;
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

constexpr int kValThreads = 256;
constexpr int kValStages = 4;       // tiles in flight per thread
constexpr int kValMaxTiles = 4096;  // tiles per CTA (their row pointers sit in shared memory)

// max_t v_scale[b, t] for each batch row (bounds every weight p_t * s_t).
__global__ void row_max_kernel(const float* __restrict__ vs, int64_t T, int64_t ld,
                               float* __restrict__ out) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  float m = 0.f;
  for (int64_t t = threadIdx.x; t < T; t += blockDim.x) m = fmaxf(m, vs[b * ld + t]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    m = warp_max(m);
    if (threadIdx.x == 0) out[b] = m;
  }
}

// Value-kernel shared memory: LUT (reused for the final lane reduction), the
// split's outlier row pointers and the cp.async ring (per stage and thread:
// 16-byte slab slot, G probabilities, scale, zero, one outlier entry).
template <int BITS, int G>
struct ValSmem {
  static constexpr int kRed = 8 * 32 * 33 * 4;
  static constexpr int kLut = PairLut<BITS>::kBytes > kRed ? PairLut<BITS>::kBytes : kRed;
  static constexpr int kPtr = kLut;
  static constexpr int kRing = kPtr + (kValMaxTiles + 1) * 4 + 12;  // 16-byte aligned
  static constexpr int kPerThread = 16 + 4 * (G + 3);  // slab + G probs + scale + zero + entry
  static constexpr int kStage = kValThreads * kPerThread;  // [slab][G probs][scale][zero][entry]
  static constexpr int kBytes = kRing + kValStages * kStage;
};

template <int BITS, int G>
__global__ void __launch_bounds__(kValThreads) value_kernel(ValueArgs a, const float* __restrict__ row_max) {
  extern __shared__ __align__(16) uint8_t smem[];
  using S = ValSmem<BITS, G>;
  uint8_t* lut = smem;
  float* red = reinterpret_cast<float*>(smem);  // after the main loop
  int32_t* tptr = reinterpret_cast<int32_t*>(smem + S::kPtr);
  __shared__ float s_acc[G][129];  // outliers + sink (fp32) and the zero term at [128]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = warp & 3, par = warp >> 2;
  const int ptid = threadIdx.x & 127;
  const uint32_t lane4 = (uint32_t)lane << 2;
  PairLut<BITS>::build(lut, a.cb);
  for (int idx = threadIdx.x; idx < G * 129; idx += blockDim.x) (&s_acc[0][0])[idx] = 0.f;

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
  const float* prow = a.probs + (b * HG + h * G) * a.T;
  // weights p_t * s_t <= max_t s_t (probabilities are <= 1): scale them so the
  // largest possible weight is 2^14 in fp16
  const float e_scale = ldexpf(1.f, 14 - pow2_exponent(row_max[b]));
  const float inv_e = 1.f / e_scale;
  for (int64_t k = threadIdx.x; k <= tb - ta; k += blockDim.x)
    tptr[k] = __ldg(a.out_ptr + u * a.nt_cap + ta + k);
  __syncthreads();

  float acc[G][32];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < 32; ++c) acc[g][c] = 0.f;
  float zsum[G];
#pragma unroll
  for (int g = 0; g < G; ++g) zsum[g] = 0.f;

  const int64_t tbytes = kTileTokens * kHeadDim * BITS / 8;
  const int64_t slab_off = (int64_t)(j * 32 + lane) * (4 * BITS);
  const uint8_t* ubase = a.codes + u * a.nt_cap * tbytes + slab_off;
  // Stage layout (structure of arrays, conflict-free): slabs [thread][16 B],
  // then 4-byte fields [G + 3][thread].
  uint8_t* ring = smem + S::kRing;
  const int fb = kValThreads * 16;  // byte offset of the 4-byte fields in a stage

  // This warp's tiles: ta + par, ta + par + 2, ...; the i-th of them goes to
  // ring stage i % kValStages.
  const int64_t t0 = ta + par;
  const int64_t my_n = t0 < tb ? (tb - t0 + 1) / 2 : 0;
  auto issue = [&](int64_t i) {
    if (i < my_n) {
      const int64_t tile = t0 + 2 * i;
      uint8_t* stage = ring + (i % kValStages) * S::kStage;
      CodeSlab<BITS>::copy(smem_u32(stage + threadIdx.x * 16), ubase + tile * tbytes, true);
      const uint32_t fdst = smem_u32(stage + fb + threadIdx.x * 4);
      const int64_t t = tile * kTileTokens + lane;
      const bool live = t < a.T && !(sink && t == 0);
      const int64_t tc = live ? t : 0;
#pragma unroll
      for (int g = 0; g < G; ++g)
        cp_async4(fdst + g * kValThreads * 4, prow + g * a.T + tc, live ? 4u : 0u);
      cp_async4(fdst + G * kValThreads * 4, vs + tc, live ? 4u : 0u);
      cp_async4(fdst + (G + 1) * kValThreads * 4, vz + tc, live ? 4u : 0u);
      const int32_t e0 = tptr[tile - ta], e1 = tptr[tile - ta + 1];
      const int32_t e = e0 + ptid;
      cp_async4(fdst + (G + 2) * kValThreads * 4, a.out_ent + (e < e1 ? e : 0), e < e1 ? 4u : 0u);
    }
    cp_async_commit();
  };

  for (int64_t i = 0; i < kValStages - 1; ++i) issue(i);
  for (int64_t i = 0; i < my_n; ++i) {
    issue(i + kValStages - 1);
    cp_async_wait<kValStages - 1>();
    const int64_t tile = t0 + 2 * i;
    const uint8_t* stage = ring + (i % kValStages) * S::kStage;
    CodeSlab<BITS> cw;
    cw.read(stage + threadIdx.x * 16);
    const float* f = reinterpret_cast<const float*>(stage + fb) + threadIdx.x;
    float w32[G];
    uint16_t w16[G];
    const float s_t = f[G * kValThreads], z_t = f[(G + 1) * kValThreads];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float p = f[g * kValThreads];
      w32[g] = p * s_t;
      const __half hw = __float2half_rn(w32[g] * e_scale);
      w16[g] = __half_as_ushort(hw);
      if (warp == 0 || warp == 4) zsum[g] = fmaf(p, z_t, zsum[g]);
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const uint32_t l = *reinterpret_cast<const uint32_t*>(lut + PairLut<BITS>::addr(cw.w, m, lane4));
      uint16_t l1, l2;
      unpack16(l, l1, l2);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        acc[g][2 * m] = fma_h(l1, w16[g], acc[g][2 * m]);
        acc[g][2 * m + 1] = fma_h(l2, w16[g], acc[g][2 * m + 1]);
      }
    }
    // Outliers: w_t * o into channel d. Every warp holds the 32 tokens' weights
    // (lane = token), so the weight of the entry's token is one shuffle away.
    const int32_t e0 = tptr[tile - ta], e1 = tptr[tile - ta + 1];
    uint32_t ent = __float_as_uint(f[(G + 2) * kValThreads]);
    for (int32_t eb = e0; eb < e1; eb += 128) {
      const int32_t e = eb + ptid;
      if (eb != e0 && e < e1) ent = __ldg(a.out_ent + e);
      const int src = (int)((ent >> 7) & 31);
      const float oval = entry_value(ent);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float wt = __shfl_sync(0xffffffffu, w32[g], src);
        if (e < e1) atomicAdd(&s_acc[g][ent & 127], wt * oval);
      }
    }
  }
  cp_async_wait<0>();
  // Sink (token 0 in the first split).
  if (sink && ta == 0 && a.T > 0) {
    for (int idx = threadIdx.x; idx < G * kHeadDim; idx += blockDim.x) {
      const int g = idx / kHeadDim, d = idx % kHeadDim;
      const float p0 = prow[g * a.T];
      atomicAdd(&s_acc[g][d], p0 * __half2float(a.v_sink[(b * a.H + h) * kHeadDim + d]));
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float z = warp_sum(zsum[g]);
    if ((warp == 0 || warp == 4) && lane == 0) atomicAdd(&s_acc[g][128], z);
  }
  // Reduce the 64 token lanes (two warps) of each chunk (channels 32j..32j+31).
#pragma unroll
  for (int g = 0; g < G; ++g) {
    __syncthreads();  // LUT reads (g == 0) / previous reduction reads are done
    float* r = red + warp * 32 * 33;
#pragma unroll
    for (int c = 0; c < 32; ++c) r[lane * 33 + c] = acc[g][c];
    __syncthreads();
    if (par == 0) {
      float sum = 0.f;
      const float* r0 = red + j * 32 * 33;
      const float* r1 = red + (j + 4) * 32 * 33;
#pragma unroll 8
      for (int l2 = 0; l2 < 32; ++l2) sum += r0[l2 * 33 + lane] + r1[l2 * 33 + lane];
      const int d = 32 * j + lane;
      float* dst = a.partial + ((int64_t)split * (U * G) + u * G + g) * 129;
      dst[d] = sum * inv_e + s_acc[g][d];
      if (threadIdx.x == 0) dst[128] = s_acc[g][128];
    }
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

inline int value_splits(int64_t U, int64_t nt, int64_t G) {
  // one full wave: 148 SMs x resident CTAs (2 for G <= 2, 1 above), but at
  // least 16 tiles per CTA and at most kValMaxTiles
  int64_t s = (148 * (G <= 2 ? 2 : 1)) / U;
  const int64_t max_s = (nt + 15) / 16;
  if (s > max_s) s = max_s;
  const int64_t min_s = (nt + kValMaxTiles - 1) / kValMaxTiles;
  if (s < min_s) s = min_s;
  if (s < 1) s = 1;
  return (int)s;
}

// ===========================================================================
// Launchers and entry points
// ===========================================================================
template <int BITS, int G>
static int launch_key(const KeyArgs& a0, cudaStream_t st) {
  KeyArgs a = a0;
  const int64_t U = a.B * a.H;
  const int UG = (int)(U < (int64_t)(kMaxSlots / G) ? U : (int64_t)(kMaxSlots / G));
  a.units_per_group = UG;
  a.n_groups = (int)((U + UG - 1) / UG);
  const int64_t nt = (a.T + kTileTokens - 1) / kTileTokens;
  const int64_t n_quads = (nt + kKeyTiles - 1) / kKeyTiles;
  a.n_items = n_quads * a.n_groups;
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
static int launch_value(const ValueArgs& a0, const float* row_max, cudaStream_t st) {
  ValueArgs a = a0;
  const int smem = ValSmem<BITS, G>::kBytes;
  cudaFuncSetAttribute(value_kernel<BITS, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int64_t U = a.B * a.H;
  value_kernel<BITS, G><<<(unsigned)(U * a.n_splits), kValThreads, smem, st>>>(a, row_max);
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
static int dispatch_value_bits(int bits, const ValueArgs& a, const float* row_max, cudaStream_t st) {
  switch (bits) {
    case 2: return launch_value<2, G>(a, row_max, st);
    case 3: return launch_value<3, G>(a, row_max, st);
    case 4: return launch_value<4, G>(a, row_max, st);
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

inline size_t softmax_ws(int64_t rows, int64_t T) {
  const int64_t nch = (T + kSoftmaxChunk - 1) / kSoftmaxChunk;
  return align256((size_t)(rows > 0 ? rows : 0) * (nch > 0 ? nch : 0) * sizeof(float2));
}

inline size_t value_ws(int64_t B, int64_t H, int64_t G, int64_t T) {
  const int64_t U = B * H;
  const int64_t nt = (T + kTileTokens - 1) / kTileTokens;
  return align256((size_t)value_splits(U, nt, G) * U * G * 129 * sizeof(float)) +
         align256((size_t)B * sizeof(float));
}

static int value_impl(const uint8_t* codes, const uint32_t* out_ent, const int32_t* out_ptr,
                      const float* v_scale, const float* v_zero, int64_t ld_stats,
                      const void* v_sink, const float* codebook, int bits, const float* probs,
                      int64_t B, int64_t H, int64_t G, int64_t T, int64_t nt_cap, void* out,
                      void* workspace, size_t workspace_bytes, cudaStream_t st) {
  int rc = check_decode_shape("value_output", B, H, G, T, nt_cap);
  if (rc) return rc;
  if (ld_stats < T) {
    set_error("value_output: ld_stats=%lld < T=%lld", (long long)ld_stats, (long long)T);
    return KVQ_ERR_INVALID;
  }
  const int64_t U = B * H;
  const int64_t nt = (T + kTileTokens - 1) / kTileTokens;
  const int n_splits = value_splits(U, nt, G);
  const size_t part_bytes = align256((size_t)n_splits * U * G * 129 * sizeof(float));
  const size_t need = part_bytes + align256((size_t)B * sizeof(float));
  if (!workspace || workspace_bytes < need) {
    set_error("value_output: workspace too small (%zu < %zu)", workspace_bytes, need);
    return KVQ_ERR_INVALID;
  }
  ValueArgs a{};
  a.codes = codes; a.out_ent = out_ent; a.out_ptr = out_ptr; a.v_scale = v_scale;
  a.v_zero = v_zero; a.ld = ld_stats; a.v_sink = (const __half*)v_sink; a.cb = codebook;
  a.probs = probs; a.B = B; a.H = H; a.G = G; a.T = T; a.nt_cap = nt_cap;
  a.n_splits = n_splits;
  a.partial = reinterpret_cast<float*>(workspace);
  float* row_max = reinterpret_cast<float*>((char*)workspace + part_bytes);
  row_max_kernel<<<(unsigned)B, 256, 0, st>>>(v_scale, T, ld_stats, row_max);
  switch (G) {
    case 1: rc = dispatch_value_bits<1>(bits, a, row_max, st); break;
    case 2: rc = dispatch_value_bits<2>(bits, a, row_max, st); break;
    case 4: rc = dispatch_value_bits<4>(bits, a, row_max, st); break;
    case 8: rc = dispatch_value_bits<8>(bits, a, row_max, st); break;
    default: rc = KVQ_ERR_UNSUPPORTED;
  }
  if (rc) return rc;
  value_combine_kernel<<<(unsigned)(U * G), kHeadDim, 0, st>>>(a.partial, n_splits, U * G,
                                                                 (__half*)out);
  return check_launch("value_output");
}

// Workspace of decode_attention: [scores][probs][softmax partials][value partials].
struct DecodeWs {
  size_t scores, probs, soft, value, total;
};
inline DecodeWs decode_ws(int64_t B, int64_t H, int64_t G, int64_t T) {
  DecodeWs w;
  const int64_t rows = B * H * G;
  w.scores = align256((size_t)rows * T * sizeof(float));
  w.probs = w.scores;
  w.soft = softmax_ws(rows, T);
  w.value = value_ws(B, H, G, T);
  w.total = w.scores + w.probs + w.soft + w.value;
  return w;
}

}  // namespace kvq

extern "C" int kvq_key_scores(const uint8_t* codes, const uint32_t* out_ent,
                              const int32_t* out_ptr, const float* k_scale, const float* k_zero,
                              const void* k_sink, const float* codebook, int bits, const void* q,
                              const float* inv_freq, int64_t B, int64_t n_heads, int64_t group,
                              int64_t T, int64_t nt_cap, float* scores, void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_decode_shape("key_scores", B, n_heads, group, T, nt_cap);
  if (rc) return rc;
  KeyArgs a{};
  a.codes = codes; a.out_ent = out_ent; a.out_ptr = out_ptr; a.k_scale = k_scale;
  a.k_zero = k_zero; a.k_sink = (const __half*)k_sink; a.cb = codebook; a.q = (const __half*)q;
  a.inv_freq = inv_freq; a.B = B; a.H = n_heads; a.G = group; a.T = T; a.nt_cap = nt_cap;
  a.scores = scores;
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
  return kvq::softmax_ws(rows, T);
}

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

extern "C" int kvq_value_output(const uint8_t* codes, const uint32_t* out_ent,
                                const int32_t* out_ptr, const float* v_scale,
                                const float* v_zero, int64_t ld_stats, const void* v_sink,
                                const float* codebook, int bits, const float* probs, int64_t B,
                                int64_t n_heads, int64_t group, int64_t T, int64_t nt_cap,
                                void* out, void* workspace, size_t workspace_bytes,
                                void* stream) {
  kvq::clear_error();
  return kvq::value_impl(codes, out_ent, out_ptr, v_scale, v_zero, ld_stats, v_sink, codebook,
                         bits, probs, B, n_heads, group, T, nt_cap, out, workspace,
                         workspace_bytes, kvq::as_stream(stream));
}

extern "C" size_t kvq_decode_attention_workspace(int64_t B, int64_t n_heads, int64_t group,
                                                 int64_t T) {
  return kvq::decode_ws(B, n_heads, group, T).total;
}

extern "C" int kvq_decode_attention(
    const uint8_t* k_codes, const uint32_t* k_out_ent, const int32_t* k_out_ptr,
    const float* k_scale, const float* k_zero, const void* k_sink, const float* k_codebook,
    const uint8_t* v_codes, const uint32_t* v_out_ent, const int32_t* v_out_ptr,
    const float* v_scale, const float* v_zero, int64_t ld_stats, const void* v_sink,
    const float* v_codebook, int bits, const void* q, const float* inv_freq, int64_t B,
    int64_t n_heads, int64_t group, int64_t T, int64_t nt_cap, void* out, float* scores_out,
    float* probs_out, void* workspace, size_t workspace_bytes, void* stream) {
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
  rc = kvq_key_scores(k_codes, k_out_ent, k_out_ptr, k_scale, k_zero, k_sink, k_codebook, bits,
                      q, inv_freq, B, n_heads, group, T, nt_cap, scores, stream);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  rc = softmax_impl(scores, B * n_heads * group, T, 0.08838834764831845f /* 1/sqrt(128) */,
                    probs, soft, w.soft, st);
  if (rc) return rc;
  return value_impl(v_codes, v_out_ent, v_out_ptr, v_scale, v_zero, ld_stats, v_sink, v_codebook,
                    bits, probs, B, n_heads, group, T, nt_cap, out, val, w.value, st);
}
