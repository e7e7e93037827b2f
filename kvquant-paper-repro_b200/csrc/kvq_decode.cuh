// Decode attention over the packed quantized cache, on the tensor cores.
//
// Key kernel: score[b,hq,t] = q . RoPE_t(Khat_t), Khat = (cb[code] + o) * s + z
// per channel (kvquant/quant/kv_quantizer.py:89), rotate-half RoPE with fp32
// angles fl(t * inv_freq) (kvquant/kernels/rope_fused.py:6-12). Per RoPE pair
// (channels p, p+64) with code values L1, L2:
//   X = L1*(s1 q1) + L2*(s2 q2) + (z1 q1 + z2 q2)
//   Y = L1*(s1 q2) - L2*(s2 q1) + (z1 q2 - z2 q1)
//   score += cos(t th_p) * X + sin(t th_p) * Y
// X and Y of 16 tokens x 4 pairs are one m16n8k8 MMA whose A operand is the
// fp16 code values read from the LUT and whose C operand is the zero-point
// term; the rotation is an fp32 epilogue; outliers come from the tile-CSR.
//
// Value kernel: out[b,hq,:] = sum_t p_t * (s_t * (cb[code] + o) + z_t) with the
// per-token scale s_t / zero z_t over all channels (kv_quantizer.py:103-117);
// the code-value x weight sum is an m16n8k16 MMA per 16 tokens x 16 channels.
//
// The packed tiles are laid out so that each lane's slab already holds the code
// pairs of its MMA fragments (A-operand order), so a lane turns one slab byte
// (4-bit) into one LUT address and the LUT word is the fragment register.
// Both kernels stream codes, per-token data and outlier entries through
// cp.async rings in shared memory.
#pragma once
#include "kvq_common.cuh"

namespace kvq {

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
};

// Pair LUT with the code values split into fp16 high and low parts (cb = hi +
// lo to ~2^-22 relative): entry v (a code pair, first code in the low bits) of
// lane l at byte (v << 8) | (l << 3) holds {half2(hi, hi), half2(lo, lo)}, so a
// lane's 8-byte lookups hit distinct bank pairs. The low parts keep the
// dequantized value exact where s * cb and the zero point nearly cancel.
template <int BITS>
struct PairLutHiLo {
  static constexpr int kEntries = 1 << (2 * BITS);
  static constexpr int kBytes = kEntries * 256;
  __device__ static void build(uint8_t* smem, const float* cb) {
    constexpr int mask = (1 << BITS) - 1;
    for (int idx = threadIdx.x; idx < kEntries * 32; idx += blockDim.x) {
      const int v = idx >> 5, lane = idx & 31;
      const float c0 = cb[v & mask], c1 = cb[v >> BITS];
      const __half h0 = __float2half_rn(c0), h1 = __float2half_rn(c1);
      const uint32_t hi = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      const uint32_t lo = half2_bits(c0 - __half2float(h0), c1 - __half2float(h1));
      *reinterpret_cast<uint2*>(smem + (v << 8) + (lane << 3)) = make_uint2(hi, lo);
    }
  }
};

// An outlier entry's value: the reference's fp16 dequantized key / value at
// its position (see outlier_entry). The decode kernels add (value - dense) *
// coefficient, dense = cb[c0] * s + z being what the code tiles hold there.
// Pair LUT with the code values' fp16 high parts at byte (v << 8) | (lane << 2)
// and their low parts 128 bytes further, so that a lane loads each of the four
// words straight into the register of the MMA operand that needs it.
template <int BITS>
struct PairLutSplit {
  static constexpr int kEntries = 1 << (2 * BITS);
  static constexpr int kBytes = kEntries * 256;
  __device__ static void build(uint8_t* smem, const float* cb) {
    constexpr int mask = (1 << BITS) - 1;
    for (int idx = threadIdx.x; idx < kEntries * 32; idx += blockDim.x) {
      const int v = idx >> 5, lane = idx & 31;
      const float c0 = cb[v & mask], c1 = cb[v >> BITS];
      const __half h0 = __float2half_rn(c0), h1 = __float2half_rn(c1);
      const uint32_t hi = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      *reinterpret_cast<uint32_t*>(smem + (v << 8) + (lane << 2)) = hi;
      *reinterpret_cast<uint32_t*>(smem + (v << 8) + 128 + (lane << 2)) =
          half2_bits(c0 - __half2float(h0), c1 - __half2float(h1));
    }
  }
};

__device__ __forceinline__ float entry_value(uint32_t ent) {
  return __half2float(__ushort_as_half((unsigned short)(ent >> 16)));
}

// cb[c0], c0 = the code of a dense 0 (the code stored at outlier positions):
// first minimum of |cb[k]| (kvquant_ops.cu:141-148 with v = 0).
__device__ __forceinline__ float dense_zero_value(const float* cb, int n) {
  float best = cb[0], bd = fabsf(cb[0]);
  for (int k = 1; k < n; ++k) {
    const float d = fabsf(cb[k]);
    if (d < bd) { bd = d; best = cb[k]; }
  }
  return best;
}

// ---------------------------------------------------------------------------
// Angle reduction for RoPE in fp32 only: a = fl(t * f) (the reference's fp32
// angle), r = a - k * 2pi with the classic three-term Cody-Waite split of 2pi
// (each step one rounded FMA; |error| < 1e-6 rad for |a| < 2^24), then the
// hardware sin/cos on [-pi, pi] (abs error < 4e-7).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float rope_reduce(int t, float f) {  // 0 <= t < 2^24
  const float a = __fmul_rn((float)t, f);
  const float k = rintf(a * 0.15915493667125702f);  // 1 / (2 pi)
  float r = fmaf(-k, 6.2831854820251465f, a);        // fl(2 pi)
  r = fmaf(-k, -1.7484555314695172e-07f, r);          // fl(2 pi - C1)
  r = fmaf(-k, -6.8604980400235275e-15f, r);          // fl(2 pi - C1 - C2)
  return r;
}

// mma.sync wrappers (fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Lane slab of one 16-token block (8*BITS bytes = 32 code pairs). In the
// cache a block is stored structure-of-arrays: region 0 = bytes 0..15 of the
// 32 lane slabs (512 B), region 1 = their remaining 8*BITS-16 bytes; in shared
// memory a slab is staged as two 16-byte slots (the second partly used).
template <int BITS>
struct LaneSlab {
  static constexpr int kBytes = 8 * BITS;
  static constexpr int kRest = 8 * BITS - 16;  // bytes of region 1 per lane
  uint32_t w[8];
  // Asynchronous copy of lane `lane`'s slab of the block at `blk` (global).
  __device__ static __forceinline__ void copy(uint32_t dst0, uint32_t dst1, const uint8_t* blk,
                                              int lane, bool valid) {
    const uint32_t n = valid ? 1u : 0u;
    cp_async16(dst0, blk + lane * 16, 16u * n);
    if (BITS == 4) cp_async16(dst1, blk + 512 + lane * 16, 16u * n);
    if (BITS == 3) cp_async8(dst1, blk + 512 + lane * 8, 8u * n);
  }
  __device__ __forceinline__ void read(const uint8_t* s0, const uint8_t* s1) {
    const uint4 v = *reinterpret_cast<const uint4*>(s0);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    if (BITS == 4) {
      const uint4 u = *reinterpret_cast<const uint4*>(s1);
      w[4] = u.x; w[5] = u.y; w[6] = u.z; w[7] = u.w;
    } else if (BITS == 3) {
      const uint2 u = *reinterpret_cast<const uint2*>(s1);
      w[4] = u.x; w[5] = u.y; w[6] = 0; w[7] = 0;
    } else {
      w[4] = w[5] = w[6] = w[7] = 0;
    }
  }
  // LUT byte address of pair slot q for this lane.
  __device__ __forceinline__ uint32_t addr(int q, uint32_t lane4) const {
    if (BITS == 4) {
      const uint32_t sel = 0x1100u | ((4u + (q & 3)) << 4);
      return prmt(lane4, w[q >> 2], sel);
    }
    return (slab_pair<BITS>(w, q) << 8) | lane4;
  }
};

// ===========================================================================
// Key kernel (tensor cores as the dot-product engine).
//
// Per 16-token block, pair block kb (4 RoPE pairs) and query head, two
// m16n8k16 MMAs compute, for the 16 tokens,
//   X_p = L1 P1 + L2 P2 + OX   (columns 0..3, pairs 4kb..4kb+3)
//   Y_p = L1 Q1 + L2 Q2 + OY   (columns 4..7)
// Code values L and constants P, Q are split into fp16 high and low parts
// (L = Lh + Ll, P = Ph + Pl to ~2^-22 relative): per-channel calibration puts
// s * cb close to -z for most entries, so s * cb and the zero point cancel and
// a single fp16 rounding of either would be amplified many times over the
// dequantized key's own fp16 rounding. The first MMA takes A columns 0..7 =
// Lh (rows = tokens, the two halves of each pair) twice against B rows 0..7 =
// Ph, Qh (block-diagonal per head) and rows 8..15 = Pl, Ql; the second takes
// A columns 0..7 = Ll against Ph, Qh plus the zero-point terms OX / OY as A
// columns 8, 9 = 256 times B rows 8, 9 = the terms / 256 split into fp16 high
// and low parts. Ll * (Pl, Ql) (~2^-22) is dropped.
// The epilogue adds cos * X + sin * Y in fp32 with the token's exact-angle
// cos/sin held in registers. Outliers add (d - dense) (cos qa + sin qb) / sigma
// per entry with exact trig (d = the entry's dequantized key, dense = the
// MMA's cb[c0] s + z there); a block's entries (ordered by token) are summed per token with a warp
// segmented scan, so every score has exactly one writer and no shared-memory
// float atomics are needed.
//
// CTA = 16 warps, one CTA per SM; a work item is (group of up to 32 query-head
// slots, 8 tiles = 256 tokens); warp w owns 16-token block w of the item for
// every unit of the group, so the cos/sin registers are computed once per
// item and reused for every unit.
// ===========================================================================
struct KeyArgs {
  const uint8_t* codes;
  const uint32_t* out_ent;
  const int32_t* out_ptr;  // CSR rows (unit, tile, 16-token block)
  const float* k_scale;    // [H*128] local channels
  const float* k_zero;
  const __half* k_sink;    // [B, H*128] or null
  const float* cb;
  const __half* q;         // [B, H*G, 128]
  const float* inv_freq;   // [64]
  int64_t B, H, G, T, nt_cap;
  float* scores;           // [B, H*G, T]
  // optional softmax partials of softmax(scores * stat_scale): per (row,
  // 256-token item) the max and the sum of exp(x - max), float2 [B*H*G, n_oct]
  float2* stats;
  float stat_scale;
  int units_per_group, n_groups;
  int64_t n_items;         // tile octets * groups
  int64_t pos0;            // position of cached token 0 (a token-range shard starts later)
};

constexpr int kKeyWarps = 16;
constexpr int kKeyThreads = kKeyWarps * 32;
constexpr int kKeyTiles = kKeyWarps / 2;             // tiles per work item
constexpr int kKeyTokens = kKeyTiles * kTileTokens;  // 256
constexpr int kKeyRows = 2 * kKeyTiles;              // CSR rows per unit and item
constexpr int kMaxSlots = 32;                        // query heads per group
constexpr int kKeyStages = 3;                        // units in flight per thread
constexpr int kBRow = 9;  // B words per (slot, kb): half2(P) x4, half2(Q) x4, zero, each
                          // as (high parts, low parts)
constexpr int kZRow = 8;  // zero-point words per (slot, kb): half2(hi, lo) of column n's term / 256
constexpr uint32_t kA256 = 0x5C005C00u;  // half2(256, 256)

// Shared memory of the key kernel: pair LUT; zero-point words per (slot, kb,
// column); B words per (slot, kb); scores [slot][256]; per-slot scale sigma;
// RoPE inverse frequencies [64]; the item's CSR row pointers per unit; the
// cp.async ring (per stage and thread: the two 16-byte halves of the lane
// slab and one entry).
template <int BITS>
struct KeySmem {
  static constexpr int kLut = PairLutSplit<BITS>::kBytes;
  static constexpr int kZ = kLut;
  static constexpr int kB = kZ + kMaxSlots * 16 * kZRow * 4;  // uint2 (high, low) B words
  static constexpr int kSc = kB + kMaxSlots * 16 * kBRow * 8;
  static constexpr int kSigma = kSc + kMaxSlots * kKeyTokens * 4;
  static constexpr int kInv = kSigma + kMaxSlots * 4;
  static constexpr int kPtr = kInv + kPairs * 4;
  static constexpr int kQh = kPtr + kMaxSlots * (kKeyRows + 1) * 4;  // [slots][128] fp16 query
  static constexpr int kISig = kQh + kMaxSlots * kHeadDim * 2;        // [slots] 1 / sigma
  static constexpr int kRing = (kISig + kMaxSlots * 4 + 15) / 16 * 16;
  static constexpr int kStage = kKeyThreads * (16 + 16 + 4);
  static constexpr int kSZ = kRing + kKeyStages * kStage;  // per thread: (scale, zero) of its entry
  static constexpr int kBytes = kSZ + kKeyThreads * 8;
  static_assert(kBytes <= 232448, "key kernel shared memory");
};

template <int BITS>
__host__ __device__ constexpr int key_smem_bytes() { return KeySmem<BITS>::kBytes; }

// m16n8k16, fp16 inputs, fp32 result with a zero accumulator input.
__device__ __forceinline__ void mma_16816_zc(float (&d)[4], uint32_t a0, uint32_t a1,
                                             uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Packed fp32 pairs (one 64-bit register pair) and the sm_100 paired FMA,
// which issues once for two fp32 FMAs.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2sum(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ void ffma2(uint64_t& acc, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

__device__ __forceinline__ float half_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float half_hi(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// Builds the per-slot tables of a group: sigma (power of two >= every |s q|
// product of the slot), zero-point words and B words, all divided by sigma.
template <int BITS, int G>
__device__ void key_build_tables(const KeyArgs& a, uint8_t* smem, int u0, int nu) {
  using L = KeySmem<BITS>;
  float* sigma = reinterpret_cast<float*>(smem + L::kSigma);
  uint32_t* zt = reinterpret_cast<uint32_t*>(smem + L::kZ);
  uint2* bt = reinterpret_cast<uint2*>(smem + L::kB);
  const int64_t HG = a.H * G;
  for (int s = threadIdx.x; s < kMaxSlots; s += blockDim.x) sigma[s] = 0.f;
  __syncthreads();
  for (int idx = threadIdx.x; idx < nu * G * kPairs; idx += blockDim.x) {
    const int s = idx / kPairs, p = idx % kPairs;
    const int64_t u = u0 + s / G;
    const int64_t b = u / a.H, h = u % a.H;
    const __half* qv = a.q + (b * HG + h * G + s % G) * kHeadDim;
    const float q1 = __half2float(qv[p]), q2 = __half2float(qv[p + 64]);
    const float s1 = a.k_scale[h * kHeadDim + p], s2 = a.k_scale[h * kHeadDim + p + 64];
    const float m = fmaxf(fmaxf(fabsf(s1 * q1), fabsf(s2 * q2)), fmaxf(fabsf(s1 * q2), fabsf(s2 * q1)));
    atomicMax(reinterpret_cast<int*>(sigma + s), __float_as_int(m));
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nu * G * 16 * (kZRow + kBRow); idx += blockDim.x) {
    const int s = idx / (16 * (kZRow + kBRow)), r = idx % (16 * (kZRow + kBRow));
    const int kb = r / (kZRow + kBRow), j = r % (kZRow + kBRow);
    const int64_t u = u0 + s / G;
    const int64_t b = u / a.H, h = u % a.H;
    const __half* qv = a.q + (b * HG + h * G + s % G) * kHeadDim;
    const float* scl = a.k_scale + h * kHeadDim;
    const float* zer = a.k_zero + h * kHeadDim;
    const float inv = ldexpf(1.f, -pow2_exponent(sigma[s]));
    if (j < kZRow) {  // zero-point word of column j: OX (j < 4) or OY of pair 4kb + (j & 3)
      const int p = 4 * kb + (j & 3);
      const float q1 = __half2float(qv[p]), q2 = __half2float(qv[p + 64]);
      const float z1 = zer[p], z2 = zer[p + 64];
      const float zt256 = (j < 4 ? (z1 * q1 + z2 * q2) : (z1 * q2 - z2 * q1)) * inv * (1.f / 256.f);
      const __half hi = __float2half_rn(zt256);
      const __half lo = __float2half_rn(zt256 - __half2float(hi));
      zt[(s * 16 + kb) * kZRow + j] = (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
    } else {      // B word jj: half2(P1, P2) of pair 4kb+jj (jj < 4), half2(Q1, Q2) of 4kb+jj-4
      const int jj = j - kZRow;
      uint32_t w = 0u, wl = 0u;
      if (jj < 8) {
        const int p = 4 * kb + (jj & 3);
        const float q1 = __half2float(qv[p]), q2 = __half2float(qv[p + 64]);
        const float s1 = scl[p], s2 = scl[p + 64];
        const float v1 = jj < 4 ? s1 * q1 * inv : s1 * q2 * inv;
        const float v2 = jj < 4 ? s2 * q2 * inv : -s2 * q1 * inv;
        const __half h1 = __float2half_rn(v1), h2 = __float2half_rn(v2);
        w = (uint32_t)__half_as_ushort(h1) | ((uint32_t)__half_as_ushort(h2) << 16);
        wl = half2_bits(v1 - __half2float(h1), v2 - __half2float(h2));
      }
      bt[(s * 16 + kb) * kBRow + jj] = make_uint2(w, wl);
    }
  }
  __syncthreads();
  if (threadIdx.x < kMaxSlots) {
    const int e = pow2_exponent(sigma[threadIdx.x]);
    sigma[threadIdx.x] = ldexpf(1.f, e);
    reinterpret_cast<float*>(smem + L::kISig)[threadIdx.x] = ldexpf(1.f, -e);
  }
  // the slots' queries (fp16) for the outlier pass
  __half* qh = reinterpret_cast<__half*>(smem + L::kQh);
  for (int idx = threadIdx.x; idx < nu * G * kHeadDim; idx += blockDim.x) {
    const int sl = idx / kHeadDim;
    const int64_t u = u0 + sl / G;
    qh[idx] = a.q[((u / a.H) * HG + (u % a.H) * G + sl % G) * kHeadDim + idx % kHeadDim];
  }
}

template <int BITS, int G>
__global__ void __launch_bounds__(kKeyThreads, 1) key_scores_kernel(KeyArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  using L = KeySmem<BITS>;
  const uint8_t* lut = smem;
  float* sc = reinterpret_cast<float*>(smem + L::kSc);        // [slots][256 tokens]
  float* sigma = reinterpret_cast<float*>(smem + L::kSigma);  // [slots]
  int32_t* uptr = reinterpret_cast<int32_t*>(smem + L::kPtr);  // [units][kKeyRows + 1]
  uint8_t* ring = smem + L::kRing;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  // B word of this lane: column g of the block-diagonal B is X of pair g
  // (g < 4) or Y of pair g - 4; lane (g, c) holds rows 2c, 2c+1 of it.
  const int jl = (g == c) ? c : ((g == c + 4) ? 4 + c : 8);
  const uint8_t* bbase = smem + L::kB + jl * 8;
  const uint8_t* zbase = smem + L::kZ + g * 4;  // zero-point word of column g
  // A columns 8, 9 = 256 (lanes c == 0 hold them), columns 10..15 = 0
  const uint32_t a23 = c == 0 ? kA256 : 0u;
  float* invf = reinterpret_cast<float*>(smem + L::kInv);
  __shared__ float s_cb0;
  PairLutSplit<BITS>::build(smem, a.cb);
  if (threadIdx.x < kPairs) invf[threadIdx.x] = a.inv_freq[threadIdx.x];
  if (threadIdx.x == 0) s_cb0 = dense_zero_value(a.cb, 1 << BITS);

  const int nt = (int)((a.T + kTileTokens - 1) / kTileTokens);
  const int n_oct = (nt + kKeyTiles - 1) / kKeyTiles;
  const int UG = a.units_per_group;
  const int64_t w0 = a.n_items * blockIdx.x / gridDim.x;
  const int64_t w1 = a.n_items * (blockIdx.x + 1) / gridDim.x;
  const int64_t HG = a.H * G;
  const int64_t tbytes = kTileTokens * kHeadDim * BITS / 8;
  const int64_t ustride = a.nt_cap * tbytes;  // bytes between units
  const int blk_off = (warp & 1) * (256 * BITS);  // this warp's block within a tile
  int cur_group = -1;

  for (int64_t w = w0; w < w1; ++w) {
    const int grp = (int)(w / n_oct);
    const int tile0 = kKeyTiles * (int)(w % n_oct);
    const int u0 = grp * UG;
    const int nu = (int)min((int64_t)UG, a.B * a.H - u0);
    __syncthreads();  // the previous item's readers are done with sc / tables
    if (grp != cur_group) {
      cur_group = grp;
      key_build_tables<BITS, G>(a, smem, u0, nu);
    }
    for (int idx = threadIdx.x; idx < nu * G * kKeyTokens; idx += blockDim.x) sc[idx] = 0.f;
    const int ntiles = min(kKeyTiles, nt - tile0);
    for (int idx = threadIdx.x; idx < nu * (kKeyRows + 1); idx += blockDim.x) {
      const int ui = idx / (kKeyRows + 1), k = idx % (kKeyRows + 1);
      uptr[idx] = __ldg(a.out_ptr + 2 * ((int64_t)(u0 + ui) * a.nt_cap + tile0) + min(k, 2 * ntiles));
    }
    __syncthreads();

    const int my_tile = tile0 + (warp >> 1);
    const bool has = my_tile < nt;
    const uint8_t* src = a.codes + ((int64_t)u0 * a.nt_cap + (has ? my_tile : tile0)) * tbytes + blk_off;
    int wr_stage = 0;
    auto issue = [&](int ui) {
      if (ui < nu) {
        uint8_t* st = ring + wr_stage * L::kStage;
        LaneSlab<BITS>::copy(smem_u32(st + threadIdx.x * 16),
                             smem_u32(st + kKeyThreads * 16 + threadIdx.x * 16), src, lane, has);
        src += ustride;
        const int32_t e0 = uptr[ui * (kKeyRows + 1) + warp], e1 = uptr[ui * (kKeyRows + 1) + warp + 1];
        const int32_t e = e0 + lane;
        cp_async4(smem_u32(st + kKeyThreads * 32 + threadIdx.x * 4), a.out_ent + (e < e1 ? e : 0),
                  e < e1 ? 4u : 0u);
        wr_stage = wr_stage == kKeyStages - 1 ? 0 : wr_stage + 1;
      }
      cp_async_commit();
    };
    for (int ui = 0; ui < kKeyStages - 1; ++ui) issue(ui);

    // cos (c < 2) or sin (c >= 2) of tokens g, g + 8 of this warp's block for
    // pairs 4kb + 2(c & 1) + {0, 1}.
    const int tok0 = (int)a.pos0 + tile0 * kTileTokens + 16 * warp;  // position of the block's first token
    // Lanes c and c ^ 2 need the same angles (one the cosines, the other the
    // sines): each evaluates one of the pair's two angles (e = c >> 1) with
    // sin and cos, keeps its own function and passes the other one across.
    const bool want_cos = c < 2;
    // tw[kb][0] = the pair (e = 0, 1) for token g, tw[kb][1] for token g + 8
    uint64_t tw[16][2];
#pragma unroll
    for (int kb = 0; kb < 16; ++kb) {
      const float f = invf[4 * kb + 2 * (c & 1) + (c >> 1)];
      float s0, c0, s8, c8;
      __sincosf(rope_reduce(tok0 + g, f), &s0, &c0);
      __sincosf(rope_reduce(tok0 + g + 8, f), &s8, &c8);
      const float k0 = want_cos ? c0 : s0, k8 = want_cos ? c8 : s8;
      const float r0 = __shfl_xor_sync(0xffffffffu, want_cos ? s0 : c0, 2);
      const float r8 = __shfl_xor_sync(0xffffffffu, want_cos ? s8 : c8, 2);
      tw[kb][0] = want_cos ? f2pack(k0, r0) : f2pack(r0, k0);
      tw[kb][1] = want_cos ? f2pack(k8, r8) : f2pack(r8, k8);
    }

    int rd_stage = 0;
    int ho = (int)(u0 % a.H);  // KV head of unit u0 + ui
    float2* szs = reinterpret_cast<float2*>(smem + L::kSZ) + threadIdx.x;
    for (int ui = 0; ui < nu; ++ui) {
      // cp.async groups per iteration: this unit's (scale, zero) pair, then the
      // ring copy kKeyStages - 1 units ahead; waiting for all but the newest
      // one therefore completes ring copy ui (and every pair before it).
      cp_async_wait<kKeyStages - 2>();
      const uint8_t* st = ring + rd_stage * L::kStage;
      rd_stage = rd_stage == kKeyStages - 1 ? 0 : rd_stage + 1;
      LaneSlab<BITS> sl;
      sl.read(st + threadIdx.x * 16, st + kKeyThreads * 16 + threadIdx.x * 16);
      const uint32_t ent0 = *reinterpret_cast<const uint32_t*>(st + kKeyThreads * 32 + threadIdx.x * 4);
      const int slot0 = ui * G;
      // Scale and zero of the channel of this lane's entry among the block's
      // first 32, fetched now so that the outlier pass after the MMA loop finds
      // them in shared memory instead of waiting on L2.
      {
        const int32_t f0 = uptr[ui * (kKeyRows + 1) + warp], f1 = uptr[ui * (kKeyRows + 1) + warp + 1];
        const bool fv = f0 + lane < f1;
        const int64_t off = fv ? (int64_t)ho * kHeadDim + (ent0 & 127) : 0;
        const uint32_t dst = smem_u32(szs);
        cp_async4(dst, a.k_scale + off, fv ? 4u : 0u);
        cp_async4(dst + 4, a.k_zero + off, fv ? 4u : 0u);
        cp_async_commit();
      }
      issue(ui + kKeyStages - 1);
      const uint8_t* brow = bbase + slot0 * (16 * kBRow * 8);
      const uint8_t* zrow = zbase + slot0 * (16 * kZRow * 4);

      uint64_t accA[G], accB[G];  // pairs of partial sums, token g / g + 8
#pragma unroll
      for (int gg = 0; gg < G; ++gg) accA[gg] = accB[gg] = 0ull;
#pragma unroll
      for (int kb = 0; kb < 16; ++kb) {
        const uint8_t* p0 = lut + sl.addr(2 * kb, lane4);
        const uint8_t* p1 = lut + sl.addr(2 * kb + 1, lane4);
        const uint32_t h0 = *reinterpret_cast<const uint32_t*>(p0);
        const uint32_t h1 = *reinterpret_cast<const uint32_t*>(p1);
        const uint32_t l0 = *reinterpret_cast<const uint32_t*>(p0 + 128);
        const uint32_t l1 = *reinterpret_cast<const uint32_t*>(p1 + 128);
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
          const uint2 bhl = *reinterpret_cast<const uint2*>(brow + (gg * 16 + kb) * (kBRow * 8));
          const uint32_t bh = bhl.x, bl = bhl.y;
          const uint32_t bz = *reinterpret_cast<const uint32_t*>(zrow + (gg * 16 + kb) * (kZRow * 4));
          float d[4], e[4];
          mma_16816_zc(d, h0, h1, l0, l1, bh, bh);    // (Lh + Ll) (Ph, Qh)
          mma_16816_zc(e, h0, h1, a23, a23, bl, bz);  // Lh (Pl, Ql) + (OX, OY)
          ffma2(accA[gg], tw[kb][0], f2add(f2pack(d[0], d[1]), f2pack(e[0], e[1])));
          ffma2(accB[gg], tw[kb][1], f2add(f2pack(d[2], d[3]), f2pack(e[2], e[3])));
        }
      }
#pragma unroll
      for (int gg = 0; gg < G; ++gg) {
        float x = f2sum(accA[gg]), y = f2sum(accB[gg]);
        x += __shfl_xor_sync(0xffffffffu, x, 1);
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        x += __shfl_xor_sync(0xffffffffu, x, 2);
        y += __shfl_xor_sync(0xffffffffu, y, 2);
        if (c == 0) {  // this warp is the only writer of its block's scores
          sc[(slot0 + gg) * kKeyTokens + 16 * warp + g] = x;
          sc[(slot0 + gg) * kKeyTokens + 16 * warp + g + 8] = y;
        }
      }
      // Outliers of the block: (d - dense) * (cos qa + sin qb) / sigma for the
      // channel's half of the pair, d the entry's dequantized key, dense =
      // cb[c0] s + z the MMA's term there, (qa, qb) = (q1, q2) for channels
      // p < 64 and (q2, -q1) for p + 64.
      const int32_t e0 = uptr[ui * (kKeyRows + 1) + warp], e1 = uptr[ui * (kKeyRows + 1) + warp + 1];
      if (e0 < e1) {
        cp_async_wait<1>();  // this unit's (scale, zero) pairs
        const __half* qrow = reinterpret_cast<const __half*>(smem + L::kQh) + slot0 * kHeadDim;
        const float* isig = reinterpret_cast<const float*>(smem + L::kISig) + slot0;
        __syncwarp();
        for (int32_t eb = e0; eb < e1; eb += 32) {
          const int32_t e = eb + lane;
          const bool valid = e < e1;
          uint32_t en = eb == e0 ? ent0 : (valid ? __ldg(a.out_ent + e) : 0u);
          const int tok = valid ? (int)((en >> 7) & 15) : 16 + lane;  // token within the block
          const int ch = (int)(en & 127), p = ch & 63;
          float sv, cv;
          __sincosf(rope_reduce(tok0 + (tok & 15), invf[p]), &sv, &cv);
          const float2 kz = eb == e0 ? *szs
                                     : make_float2(a.k_scale[(int64_t)ho * kHeadDim + ch],
                                                   a.k_zero[(int64_t)ho * kHeadDim + ch]);
          const float ov = valid ? entry_value(en) - fmaf(s_cb0, kz.x, kz.y) : 0.f;
          // Entries are ordered by token: suffix sums within runs of equal
          // tokens; runs are almost always at most 4 long (two steps), longer
          // ones take the remaining steps.
          const int tn1 = __shfl_down_sync(0xffffffffu, tok, 1);
          const int tn2 = __shfl_down_sync(0xffffffffu, tok, 2);
          const int tn4 = __shfl_down_sync(0xffffffffu, tok, 4);
          const int tprev = __shfl_up_sync(0xffffffffu, tok, 1);  // every lane takes part
          const bool head = valid && (lane == 0 || tprev != tok);
          const bool longer = __any_sync(0xffffffffu, head && lane + 4 < 32 && tn4 == tok);
#pragma unroll
          for (int gg = 0; gg < G; ++gg) {
            const float q1 = __half2float(qrow[gg * kHeadDim + p]);
            const float q2 = __half2float(qrow[gg * kHeadDim + p + 64]);
            const float qa = ch >= 64 ? q2 : q1, qb = ch >= 64 ? -q1 : q2;
            float v = ov * fmaf(cv, qa, sv * qb) * isig[gg];
            float o = __shfl_down_sync(0xffffffffu, v, 1);
            if (lane + 1 < 32 && tn1 == tok) v += o;
            o = __shfl_down_sync(0xffffffffu, v, 2);
            if (lane + 2 < 32 && tn2 == tok) v += o;
            if (longer) {
#pragma unroll
              for (int sh = 4; sh < 32; sh <<= 1) {
                const int tn = __shfl_down_sync(0xffffffffu, tok, sh);
                o = __shfl_down_sync(0xffffffffu, v, sh);
                if (lane + sh < 32 && tn == tok) v += o;
              }
            }
            if (head) sc[(slot0 + gg) * kKeyTokens + 16 * warp + tok] += v;
          }
          __syncwarp();
        }
      }
      ho = ho + 1 == (int)a.H ? 0 : ho + 1;
    }
    cp_async_wait<0>();
    __syncthreads();

    // Sink token (position 0, no rotation): score = q . k_sink, fp32.
    if (tile0 == 0 && a.k_sink) {
      for (int s = warp; s < nu * G; s += kKeyWarps) {
        const int64_t u = u0 + s / G;
        const int64_t b = u / a.H, h = u % a.H;
        const __half* qv = a.q + (b * HG + h * G + s % G) * kHeadDim;
        const __half* kv = a.k_sink + (b * a.H + h) * kHeadDim;
        float v = 0.f;
        for (int dd = lane; dd < kHeadDim; dd += 32) v = fmaf(__half2float(qv[dd]), __half2float(kv[dd]), v);
        v = warp_sum(v);
        if (lane == 0) sc[s * kKeyTokens] = v / sigma[s];
      }
      __syncthreads();
    }

    // Scores of the item, one warp per (slot, 32-token chunk) (row u * G + gg =
    // u0 * G + s), so that items of few slots still use every warp, and the
    // item's softmax partials of scores * stat_scale when asked for.
    {
      const int nvalid = (int)min((int64_t)kKeyTokens, a.T - (int64_t)tile0 * kTileTokens);
      const float f = a.stat_scale;
      constexpr int kChunks = kKeyTokens / 32;
      const int64_t nblk = (a.T + 15) / 16;
      const int64_t b0 = (int64_t)tile0 * kTileTokens / 16;
      for (int idx = warp; idx < nu * G * kChunks; idx += kKeyWarps) {
        const int sl = idx / kChunks, k = idx % kChunks;
        const int64_t row = (int64_t)u0 * G + sl;
        const int tt = lane + 32 * k;
        const float x = sc[sl * kKeyTokens + tt] * sigma[sl];
        if (tt < nvalid) a.scores[row * a.T + (int64_t)tile0 * kTileTokens + tt] = x;
        if (a.stats) {
          // partials per 16-token block (lanes 0-15 / 16-31), with the same
          // rounding as the value kernel's (score * scale) on the stored score
          const bool valid = tt < nvalid;
          const float v = valid ? x * f : -INFINITY;
          float m = v;
#pragma unroll
          for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          float l = valid ? __expf(v - m) : 0.f;
#pragma unroll
          for (int o = 1; o < 16; o <<= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
          if ((lane & 15) == 0 && 32 * k + (lane & 16) < nvalid)
            a.stats[row * nblk + b0 + 2 * k + (lane >> 4)] = make_float2(m, l);
        }
      }
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
// Value kernel (tensor cores as the weighted-sum engine).
//
// For one 16-token block and channel block mb (16 channels), one m16n8k16
// MMA accumulates D[channel][head] += sum_t cb[code(t, channel)] * w[head][t]
// with A = the fp16 code values straight from the pair LUT (rows = channels,
// k = tokens: slot q = 4 mb + i of the lane slab is fragment register a_i),
// B = the fp16 token weights w = p * s * 2^e (rows = tokens, columns = the
// query heads of the KV head, zero beyond the group) and fp32 accumulators.
// The zero-point term sum_t p_t z_t, the outliers (p s o into one channel)
// and the sink token are added in fp32 beside it; outliers go to per-warp
// accumulators (groups of up to 4 heads) so that warps do not contend.
//
// CTA = 16 warps, one CTA per SM; a work item is (unit, split of its tiles)
// and warp w takes the split's tiles w, w + 16, ...; each warp streams whole
// tiles (codes, scale/zero pairs, probabilities, outlier entries) through its
// own cp.async ring.
// ===========================================================================
struct ValueArgs {
  const uint8_t* codes;
  const uint32_t* out_ent;
  const int32_t* out_ptr;  // CSR rows (unit, tile, 16-token block)
  const float* v_scale;    // [B, ld]
  const float* v_zero;
  int64_t ld;
  const __half* v_sink;    // [B, H*128] or null
  const float* cb;
  const float* probs;      // [B, H*G, T] probabilities, or raw scores when stats is set
  // optional: per row (M, 1/L) of softmax(scores * stat_scale), merged from
  // the key kernel's partials; probs then holds raw scores and
  // p = exp(score * stat_scale - M) / L is formed here
  const float2* ml;        // [B*H*G]
  float stat_scale;
  int64_t B, H, G, T, nt_cap;
  int n_splits;
  float* partial;          // [n_splits, B*H*G, 129]: 128 channels + zero term
};

constexpr int kValWarps = 16;
constexpr int kValThreads = kValWarps * 32;
constexpr int kValMaxTiles = 2048;     // tiles per work item (row pointers sit in shared memory)
constexpr int kValSmemLimit = 232448 - 1024;  // opt-in shared memory per CTA, less static data

// max_t v_scale[b, t] for each batch row (bounds every weight p_t * s_t).
// grid = (chunks of the token axis, B); out[b] starts at 0 and takes the
// maximum by an integer atomicMax on the float bits (scales are >= 0).
constexpr int kRowMaxChunk = 16384;
__global__ void __launch_bounds__(256) row_max_kernel(const float* __restrict__ vs, int64_t T,
                                                      int64_t ld, float* __restrict__ out) {
  __shared__ float red[8];
  const int64_t b = blockIdx.y;
  const int64_t s0 = (int64_t)blockIdx.x * kRowMaxChunk, s1 = min(T, s0 + kRowMaxChunk);
  float m = 0.f;
  for (int64_t t = s0 + threadIdx.x; t < s1; t += blockDim.x) m = fmaxf(m, vs[b * ld + t]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    m = warp_max(m);
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(out + b), __float_as_int(m));
  }
}

// (max, sum of exp(x - max)) pairs merged: the pair of the union.
__device__ __forceinline__ float2 ml_merge(float2 a, float2 b) {
  const float m = fmaxf(a.x, b.x);
  if (m == -INFINITY) return a;
  return make_float2(m, a.y * __expf(a.x - m) + b.y * __expf(b.x - m));
}

// Softmax partials folded by one merge block of value_prep_kernel (256 threads x 8).
constexpr int kMlChunk = 2048;

// row_max_kernel for blockIdx.y < B. Blocks with y >= B merge the key
// kernel's softmax partials stats[row, 0..n_oct): work item (row, c) folds
// the chunk stats[row, c*kMlChunk ..) into part[row*n_mc + c]; the block that
// completes a row's last chunk (counted in count[row], zero at launch) folds
// the row's n_mc chunk pairs into ml[row] = (M, 1/L). Nothing waits on
// another block: the count only elects the block that finishes the row.
__global__ void __launch_bounds__(256) value_prep_kernel(const float* __restrict__ vs, int64_t T,
                                                         int64_t ld, float* __restrict__ out,
                                                         int64_t B,
                                                         const float2* __restrict__ stats,
                                                         int n_oct, int64_t rows, int n_mc,
                                                         float2* part, unsigned* count,
                                                         float2* __restrict__ ml) {
  __shared__ float red[8];
  __shared__ float2 red2[8];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if ((int64_t)blockIdx.y < B) {
    const int64_t b = blockIdx.y;
    const int64_t s0 = (int64_t)blockIdx.x * kRowMaxChunk, s1 = min(T, s0 + kRowMaxChunk);
    float m = 0.f;
    for (int64_t t = s0 + threadIdx.x; t < s1; t += blockDim.x) m = fmaxf(m, vs[b * ld + t]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
      m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      m = warp_max(m);
      if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(out + b), __float_as_int(m));
    }
    return;
  }
  const int64_t nb = (int64_t)gridDim.x * (gridDim.y - B);
  const int64_t items = rows * n_mc;
  for (int64_t w = blockIdx.x + (int64_t)gridDim.x * (blockIdx.y - B); w < items; w += nb) {
    const int64_t r = w / n_mc;
    const int c = (int)(w - r * n_mc);
    const float2* src = stats + r * n_oct;
    const int k1 = min(n_oct, (c + 1) * kMlChunk);
    float2 v[kMlChunk / 256];
#pragma unroll
    for (int i = 0; i < kMlChunk / 256; ++i) {
      const int k = c * kMlChunk + i * 256 + (int)threadIdx.x;
      v[i] = k < k1 ? src[k] : make_float2(-INFINITY, 0.f);
    }
    float m = v[0].x;
#pragma unroll
    for (int i = 1; i < kMlChunk / 256; ++i) m = fmaxf(m, v[i].x);
    float l = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int i = 0; i < kMlChunk / 256; ++i) l += v[i].y * __expf(v[i].x - m);
    }
    float2 acc = make_float2(m, l);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float2 other;
      other.x = __shfl_xor_sync(0xffffffffu, acc.x, o);
      other.y = __shfl_xor_sync(0xffffffffu, acc.y, o);
      acc = ml_merge(acc, other);
    }
    if (lane == 0) red2[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float2 t = red2[0];
      for (int q = 1; q < (int)(blockDim.x >> 5); ++q) t = ml_merge(t, red2[q]);
      if (n_mc == 1) {
        ml[r] = make_float2(t.x, 1.f / t.y);
        s_last = 0;
      } else {
        part[w] = t;
        __threadfence();
        s_last = atomicAdd(count + r, 1u) == (unsigned)(n_mc - 1);
      }
    }
    __syncthreads();
    if (s_last) {  // every other chunk pair of this row is visible in L2
      __threadfence();
      float2 t = make_float2(-INFINITY, 0.f);
      for (int k = threadIdx.x; k < n_mc; k += blockDim.x) t = ml_merge(t, __ldcg(part + r * n_mc + k));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float2 other;
        other.x = __shfl_xor_sync(0xffffffffu, t.x, o);
        other.y = __shfl_xor_sync(0xffffffffu, t.y, o);
        t = ml_merge(t, other);
      }
      if (lane == 0) red2[warp] = t;
      __syncthreads();
      if (threadIdx.x == 0) {
        float2 u = red2[0];
        for (int q = 1; q < (int)(blockDim.x >> 5); ++q) u = ml_merge(u, red2[q]);
        ml[r] = make_float2(u.x, 1.f / u.y);
      }
    }
    __syncthreads();
  }
}

// Value-kernel shared memory: pair LUT; fp32 outlier accumulators
// ([warp][G][128] for G <= 4, else one [G][128]); zero-term sums [G]; the
// warps' fp16 token weights of the current tile; the item's tile row
// pointers; the per-warp cp.async rings. A ring stage of one warp holds one
// tile: the two blocks' lane slabs (first 16 bytes of every lane, then the
// rest), (scale, zero) pairs [32], probabilities [G][kPRow], entries [32].
template <int BITS, int G>
struct ValSmem {
  static constexpr bool kWarpAcc = G <= 2;  // per-warp outlier sums (shared by all warps above)
  static constexpr int kLut = PairLutHiLo<BITS>::kBytes;
  static constexpr int kAcc = kLut;
  static constexpr int kAccFloats = (kWarpAcc ? kValWarps : 1) * G * kHeadDim;
  static constexpr int kZ = kAcc + kAccFloats * 8;  // outlier sums: 64-bit fixed point
  static constexpr int kW = kZ + 64;  // fp16 token weights [warp][2G][32]: high parts, low parts
  static constexpr int kPtr = kW + kValWarps * 2 * G * 64;
  // ring and stages on 128-byte boundaries, so that a warp's 512-byte copies
  // cover whole shared-memory lines
  static constexpr int kRing = (kPtr + (kValMaxTiles + 4) * 4 + 127) / 128 * 128;
  static constexpr int kBlockSlab = 1024;
  static constexpr int kSZ = 2 * kBlockSlab;
  static constexpr int kP = kSZ + 32 * 8;
  static constexpr int kPRow = 32;  // floats per probability row
  static constexpr int kE = kP + G * kPRow * 4;
  static constexpr int kStage = (kE + 32 * 4 + 127) / 128 * 128;
  static constexpr int kFit = (kValSmemLimit - kRing) / (kValWarps * kStage);
  static constexpr int kStages = kFit < 4 ? kFit : 4;
  static constexpr int kBytes = kRing + kStages * kValWarps * kStage;
  static_assert(kStages >= 2, "value ring needs two stages");
  static_assert(kStage % 128 == 0 && kRing % 128 == 0, "128-byte aligned stages");
  static_assert(kStages * kValWarps * kStage >= kValWarps * G * kHeadDim * 4,
                "the reduction buffer reuses the ring");
};

template <int BITS, int G>
__global__ void __launch_bounds__(kValThreads, 1)
    value_kernel(ValueArgs a, const float* __restrict__ row_max) {
  extern __shared__ __align__(16) uint8_t smem[];
  using S = ValSmem<BITS, G>;
  const uint8_t* lut = smem;
  unsigned long long* acc = reinterpret_cast<unsigned long long*>(smem + S::kAcc);
  float* zacc = reinterpret_cast<float*>(smem + S::kZ);
  int32_t* tptr = reinterpret_cast<int32_t*>(smem + S::kPtr);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const uint32_t lane8 = (uint32_t)lane << 3;
  unsigned long long* wacc = acc + (S::kWarpAcc ? warp * G * kHeadDim : 0);
  PairLutHiLo<BITS>::build(smem, a.cb);
  __shared__ float s_cb0;
  if (threadIdx.x == 0) s_cb0 = dense_zero_value(a.cb, 1 << BITS);
  for (int idx = threadIdx.x; idx < S::kAccFloats; idx += blockDim.x) acc[idx] = 0ull;
  if (threadIdx.x < G) zacc[threadIdx.x] = 0.f;

  const int nt = (int)((a.T + kTileTokens - 1) / kTileTokens);
  const int T = (int)a.T;
  const int64_t U = a.B * a.H;
  const int64_t u = blockIdx.x / a.n_splits;
  const int split = (int)(blockIdx.x % a.n_splits);
  const int tpb = (nt + a.n_splits - 1) / a.n_splits;
  const int ta = split * tpb, tb = min(nt, ta + tpb);
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
  // Outlier terms p (d - dense) are at most about max_t s_t (|n| <= 1 for values):
  // summed as integers in units of 2^(e - 40), e = exponent of that maximum
  // (native 64-bit shared-memory integer adds instead of float compare-and-swap
  // loops; exact, and far below 2^63 for any token count below 2^22).
  const float fix = ldexpf(1.f, min(100, max(-100, 40 - pow2_exponent(row_max[b]))));
  for (int k = threadIdx.x; k <= tb - ta; k += blockDim.x)
    tptr[k] = __ldg(a.out_ptr + 2 * (u * a.nt_cap + ta + k));
  // Softmax of raw scores: (M, 1/L) of each head of the unit.
  __shared__ float2 s_ml[8];
  if (a.ml && threadIdx.x < G) s_ml[threadIdx.x] = a.ml[b * HG + h * G + threadIdx.x];
  __syncthreads();

  // d: the weights' high parts (G <= 4: columns 4..4+G-1 hold their low parts);
  // d2 (G = 8): the low parts
  constexpr bool kSplitB = G > 4;
  float d[8][4], d2[kSplitB ? 8 : 1][4];
#pragma unroll
  for (int mb = 0; mb < 8; ++mb) d[mb][0] = d[mb][1] = d[mb][2] = d[mb][3] = 0.f;
#pragma unroll
  for (int mb = 0; mb < (kSplitB ? 8 : 1); ++mb) d2[mb][0] = d2[mb][1] = d2[mb][2] = d2[mb][3] = 0.f;
  float zs[G];
#pragma unroll
  for (int hd = 0; hd < G; ++hd) zs[hd] = 0.f;
  __half* wbuf = reinterpret_cast<__half*>(smem + S::kW) + warp * 2 * G * 32;

  const int64_t tbytes = kTileTokens * kHeadDim * BITS / 8;
  const uint8_t* src = a.codes + (u * a.nt_cap + ta + warp) * tbytes;
  int tnext = (ta + warp) * kTileTokens + lane;  // this lane's token of the next tile
  uint8_t* wring = smem + S::kRing + warp * S::kStage;
  constexpr int kStride = kValWarps * S::kStage;
  const int my_n = ta + warp < tb ? (tb - ta - warp + kValWarps - 1) / kValWarps : 0;
  int wr = 0;
  auto issue = [&](int i) {
    if (i < my_n) {
      uint8_t* st = wring + wr * kStride;
      wr = wr == S::kStages - 1 ? 0 : wr + 1;
#pragma unroll
      for (int blk = 0; blk < 2; ++blk)
        LaneSlab<BITS>::copy(smem_u32(st + blk * S::kBlockSlab + lane * 16),
                             smem_u32(st + blk * S::kBlockSlab + 512 + lane * 16),
                             src + blk * (256 * BITS), lane, true);
      src += kValWarps * tbytes;
      const int t = tnext;
      tnext += kValWarps * kTileTokens;
      const bool live = t < T && !(sink && t == 0);
      const int tc = live ? t : 0;
      const uint32_t n = live ? 4u : 0u;
      const uint32_t fsz = smem_u32(st + S::kSZ + lane * 8);
      cp_async4(fsz, vs + tc, n);
      cp_async4(fsz + 4, vz + tc, n);
#pragma unroll
      for (int hd = 0; hd < G; ++hd)
        cp_async4(smem_u32(st + S::kP + (hd * S::kPRow + lane) * 4), prow + hd * a.T + tc, n);
      const int k = warp + i * kValWarps;
      const int32_t e0 = tptr[k], e1 = tptr[k + 1];
      const int32_t e = e0 + lane;
      cp_async4(smem_u32(st + S::kE + lane * 4), a.out_ent + (e < e1 ? e : 0), e < e1 ? 4u : 0u);
    }
    cp_async_commit();
  };

  for (int i = 0; i < S::kStages - 1; ++i) issue(i);
  int rd = 0;
  for (int i = 0; i < my_n; ++i) {
    __syncwarp();  // every lane is done with the stage the next copy overwrites
    issue(i + S::kStages - 1);
    cp_async_wait<S::kStages - 1>();
    __syncwarp();  // ... and sees the other lanes' copies of this one
    const uint8_t* st = wring + rd * kStride;
    rd = rd == S::kStages - 1 ? 0 : rd + 1;
    const float2* sz = reinterpret_cast<const float2*>(st + S::kSZ);
    const float* fp = reinterpret_cast<const float*>(st + S::kP);
    // Lane = token of the tile: its weights p * s * 2^e (one per head) go to
    // the warp's fp16 weight buffer once; its zero-point terms p * z stay in
    // fp32 registers.
    {
      const float2 szl = sz[lane];
      const int tok = (ta + warp + i * kValWarps) * kTileTokens + lane;
      const bool live = tok < T && !(sink && tok == 0);
#pragma unroll
      for (int hd = 0; hd < G; ++hd) {
        float p = fp[hd * S::kPRow + lane];
        if (a.ml) {  // raw score -> probability, in place for the outlier path
          p = live ? __expf(p * a.stat_scale - s_ml[hd].x) * s_ml[hd].y : 0.f;
          const_cast<float*>(fp)[hd * S::kPRow + lane] = p;
        }
        zs[hd] = fmaf(p, szl.y, zs[hd]);
        const float wv = p * szl.x * e_scale;
        const __half wh = __float2half_rn(wv);
        wbuf[hd * 32 + lane] = wh;
        wbuf[(G + hd) * 32 + lane] = __float2half_rn(wv - __half2float(wh));
      }
    }
    __syncwarp();
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      LaneSlab<BITS> sl;
      sl.read(st + blk * S::kBlockSlab + lane * 16, st + blk * S::kBlockSlab + 512 + lane * 16);
      // B fragment of column g: weights of tokens 2c, 2c+1 (b0) and 2c+8, 2c+9 (b1).
      // G <= 4: column g < 4 = head g's high parts, column 4 + h = head h's low
      // parts; G = 8: column g = head g, high parts in (b0, b1), low in (l0, l1).
      uint32_t b0 = 0u, b1 = 0u, l0 = 0u, l1 = 0u;
      {
        const int row = kSplitB ? g : (g < 4 ? (g < G ? g : -1) : (g - 4 < G ? G + g - 4 : -1));
        if (row >= 0) {
          const __half* wg = wbuf + row * 32 + 16 * blk + 2 * c;
          b0 = *reinterpret_cast<const uint32_t*>(wg);
          b1 = *reinterpret_cast<const uint32_t*>(wg + 8);
        }
        if (kSplitB) {
          const __half* wl = wbuf + (G + g) * 32 + 16 * blk + 2 * c;
          l0 = *reinterpret_cast<const uint32_t*>(wl);
          l1 = *reinterpret_cast<const uint32_t*>(wl + 8);
        }
      }
#pragma unroll
      for (int mb = 0; mb < 8; ++mb) {
        // code values split into fp16 high and low parts: the low parts keep
        // the dequantized value exact where s * cb and the zero point cancel
        uint32_t ah[4], al[4];
#pragma unroll
        for (int ii = 0; ii < 4; ++ii) {
          const uint2 e = *reinterpret_cast<const uint2*>(lut + sl.addr(4 * mb + ii, lane8));
          ah[ii] = e.x;
          al[ii] = e.y;
        }
        mma_16816(d[mb], ah, b0, b1);
        mma_16816(d[mb], al, b0, b1);
        if (kSplitB) mma_16816(d2[kSplitB ? mb : 0], ah, l0, l1);
      }
    }
    // Outliers: p (d - dense) into channel ch, fp32; d = the entry's
    // dequantized value, dense = cb[c0] s + z the code tile's value there.
    const int k = warp + i * kValWarps;
    const int32_t e0 = tptr[k], e1 = tptr[k + 1];
    const uint32_t* fe = reinterpret_cast<const uint32_t*>(st + S::kE);
    for (int32_t eb = e0; eb < e1; eb += 32) {
      const int32_t e = eb + lane;
      if (e < e1) {
        const uint32_t en = eb == e0 ? fe[lane] : __ldg(a.out_ent + e);
        const int tok = (int)((en >> 7) & 31), ch = (int)(en & 127);
        const float so = entry_value(en) - fmaf(s_cb0, sz[tok].x, sz[tok].y);
#pragma unroll
        for (int hd = 0; hd < G; ++hd)
          atomicAdd(wacc + hd * kHeadDim + ch,
                    (unsigned long long)__float2ll_rn(fp[hd * S::kPRow + tok] * so * fix));
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int hd = 0; hd < G; ++hd) {
    const float z = warp_sum(zs[hd]);
    if (lane == 0) atomicAdd(zacc + hd, z);
  }
  __syncthreads();  // all warps are done with their rings and accumulators
  float* red = reinterpret_cast<float*>(smem + S::kRing);  // [warp][G][128]
#pragma unroll
  for (int mb = 0; mb < 8; ++mb) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (kSplitB) {
        d[mb][i] += d2[kSplitB ? mb : 0][i];
      } else {  // add the low-part columns (lanes c + 2) to the high-part ones
        d[mb][i] += __shfl_xor_sync(0xffffffffu, d[mb][i], 2);
      }
    }
  }
#pragma unroll
  for (int mb = 0; mb < 8; ++mb) {
    const int ch = 16 * mb + g;
    if (2 * c < G) {
      red[(warp * G + 2 * c) * kHeadDim + ch] = d[mb][0];
      red[(warp * G + 2 * c) * kHeadDim + ch + 8] = d[mb][2];
    }
    if (2 * c + 1 < G) {
      red[(warp * G + 2 * c + 1) * kHeadDim + ch] = d[mb][1];
      red[(warp * G + 2 * c + 1) * kHeadDim + ch + 8] = d[mb][3];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * kHeadDim; idx += blockDim.x) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kValWarps; ++w) sum += red[w * G * kHeadDim + idx];
    long long isum = 0;
    if (S::kWarpAcc) {
#pragma unroll
      for (int w = 0; w < kValWarps; ++w) isum += (long long)acc[w * G * kHeadDim + idx];
    } else {
      isum = (long long)acc[idx];
    }
    float side = (float)isum / fix;
    const int hd = idx / kHeadDim, dd = idx % kHeadDim;
    if (sink && ta == 0) {  // the sink (token 0, in the first split): p_0 * v_sink, fp32
      float p0 = prow[hd * a.T];
      if (a.ml) p0 = __expf(p0 * a.stat_scale - s_ml[hd].x) * s_ml[hd].y;
      side = fmaf(p0, __half2float(a.v_sink[(b * a.H + h) * kHeadDim + dd]), side);
    }
    float* dst = a.partial + ((int64_t)split * (U * G) + u * G + hd) * 129;
    dst[dd] = fmaf(sum, inv_e, side);
    if (dd == 0) dst[128] = zacc[hd];
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

// Merge of token-range shards of one decode step: shard i produced o_i (its
// tokens' softmax-weighted values, normalized by its own L_i) and the row's
// (M_i, 1/L_i) of softmax(scores * scale). The whole row's output is
// sum_i w_i o_i / sum_i w_i with w_i = L_i exp(M_i - M), M = max_i M_i.
__global__ void merge_shards_kernel(const __half* __restrict__ o, const float2* __restrict__ ml,
                                    int64_t n, int64_t rows, __half* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const int d = threadIdx.x;  // 128 threads
  float m = -INFINITY;
  for (int64_t i = 0; i < n; ++i) m = fmaxf(m, ml[i * rows + row].x);
  float num = 0.f, den = 0.f;
  for (int64_t i = 0; i < n; ++i) {
    const float2 p = ml[i * rows + row];
    const float w = __expf(p.x - m) / p.y;
    num = fmaf(w, __half2float(o[(i * rows + row) * kHeadDim + d]), num);
    den += w;
  }
  out[row * kHeadDim + d] = __float2half_rn(num / den);
}

// Splits of each unit's tiles into value work items. The value kernel runs
// one 16-warp CTA per SM (16 tiles in flight), so the items run in waves of
// kValSlots; the split count minimises waves x (tile rounds per warp + a
// pipeline fill of two rounds), subject to at most kValMaxTiles tiles per
// item. Host-only and independent of the device, so the workspace size is
// known up front.
constexpr int kValSlots = 148;  // B200 SMs
inline int value_splits(int64_t U, int64_t nt, int64_t /*G*/) {
  if (U < 1 || nt < 1) return 1;
  const int64_t s_min = (nt + kValMaxTiles - 1) / kValMaxTiles;
  int64_t s_max = nt / (2 * kValWarps);
  if (s_max < s_min) s_max = s_min;
  if (s_max > 4096) s_max = s_min > 4096 ? s_min : 4096;
  int64_t best = s_min, best_cost = INT64_MAX;
  for (int64_t s = s_min; s <= s_max; ++s) {
    const int64_t waves = (U * s + kValSlots - 1) / kValSlots;
    const int64_t tiles = (nt + s - 1) / s;
    const int64_t rounds = (tiles + kValWarps - 1) / kValWarps;
    const int64_t cost = waves * (rounds + 2);
    if (cost < best_cost) { best_cost = cost; best = s; }
  }
  return (int)best;
}

// Softmax partials of the key kernels: float2 [rows, key_items(T)], one per
// 16-token block: (max of score * scale, sum of exp(score * scale - max)).
inline int64_t key_items(int64_t T) { return (T + 15) / 16; }

}  // namespace kvq

#include "kvq_key_tc.cuh"
#include "kvq_value_tc.cuh"

namespace kvq {

// ===========================================================================
// Launchers and entry points
// ===========================================================================
template <int BITS, int G>
static int launch_key(const KeyArgs& a0, cudaStream_t st) {
  KeyArgs a = a0;
  const int64_t U = a.B * a.H;
  const int64_t nt = (a.T + kTileTokens - 1) / kTileTokens;
  const int64_t n_oct = (nt + kKeyTiles - 1) / kKeyTiles;
  // Units per work item. An item costs about UG unit passes plus 0.75 of one for
  // its RoPE twiddles (shared by its units), and the persistent CTAs (one per SM)
  // take the items in rounds: pick the group size that minimises rounds x item
  // cost, e.g. 32 units at 1M tokens (28 rounds) but 16 at 128K tokens (7 rounds
  // of half-size items instead of 4 rounds of full ones, the last one mostly idle).
  const int64_t ug_max = U < (int64_t)(kMaxSlots / G) ? U : (int64_t)(kMaxSlots / G);
  int64_t UG = ug_max;
  double best = 1e300;
  for (int64_t ug = ug_max; ug >= 1; --ug) {
    const int64_t groups = (U + ug - 1) / ug;
    if (groups * ug - U >= ug) continue;  // a group size that leaves an empty group
    const int64_t rounds = (n_oct * groups + kValSlots - 1) / kValSlots;
    const double cost = (double)rounds * ((double)((U + groups - 1) / groups) + 0.75);
    if (cost < best * 0.999) { best = cost; UG = (U + groups - 1) / groups; }
  }
  a.units_per_group = (int)UG;
  a.n_groups = (int)((U + UG - 1) / UG);
  a.n_items = n_oct * a.n_groups;
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
  if (G == 1 && use_key_tc()) {
    switch (bits) {
      case 2: return launch_key_tc<2>(a, st);
      case 3: return launch_key_tc<3>(a, st);
      case 4: return launch_key_tc<4>(a, st);
    }
  }
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
  if (use_value_tc()) {
    switch (bits) {
      case 2: return launch_value_tc<2, G>(a, row_max, st);
      case 3: return launch_value_tc<3, G>(a, row_max, st);
      case 4: return launch_value_tc<4, G>(a, row_max, st);
    }
  }
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
  if (B < 1 || B > 65535 || H < 1 || T < 1 || nt_cap * kTileTokens < T) {
    set_error("%s: invalid shape B=%lld H=%lld T=%lld nt_cap=%lld", what, (long long)B,
              (long long)H, (long long)T, (long long)nt_cap);
    return KVQ_ERR_INVALID;
  }
  if (!(G == 1 || G == 2 || G == 4 || G == 8)) {
    set_error("%s: group (query heads per KV head) must be 1, 2, 4 or 8 (got %lld)", what,
              (long long)G);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (T > (1LL << 24)) {  // positions are exact fp32 integers up to 2^24
    set_error("%s: T=%lld exceeds 2^24 tokens", what, (long long)T);
    return KVQ_ERR_INVALID;
  }
  return KVQ_OK;
}

// Bit width, then the code tiles' address: the kernels stage code tiles with
// 16-byte cp.async copies.
static int check_codes_aligned(const char* what, const void* codes, int bits) {
  if (bits < 2 || bits > 4) {
    set_error("%s: bits must be 2, 3 or 4 (got %d)", what, bits);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (!codes || ((uintptr_t)codes & 15u)) {
    set_error("%s: codes must be a 16-byte aligned device pointer (got %p)", what, codes);
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

// Value-path workspace: [split partials][row maxima [B] + softmax merge counts [B*H*G]].
inline size_t value_ws(int64_t B, int64_t H, int64_t G, int64_t T) {
  const int64_t U = B * H;
  const int64_t nt = (T + kTileTokens - 1) / kTileTokens;
  return align256((size_t)value_splits(U, nt, G) * U * G * 129 * sizeof(float)) +
         align256((size_t)B * sizeof(float) + (size_t)U * G * sizeof(unsigned));
}
inline int64_t ml_chunks(int64_t T) { return (key_items(T) + kMlChunk - 1) / kMlChunk; }
// ... of the raw-score variant: plus the merged (M, 1/L) per row and the
// merge's chunk pairs [B*H*G, ml_chunks(T)].
inline size_t value_scores_ws(int64_t B, int64_t H, int64_t G, int64_t T) {
  const size_t rows = (size_t)(B * H * G > 0 ? B * H * G : 0);
  return value_ws(B, H, G, T) + align256(rows * sizeof(float2)) +
         align256(rows * (size_t)ml_chunks(T > 0 ? T : 1) * sizeof(float2));
}

static int value_impl(const uint8_t* codes, const uint32_t* out_ent, const int32_t* out_ptr,
                      const float* v_scale, const float* v_zero, int64_t ld_stats,
                      const void* v_sink, const float* codebook, int bits, const float* probs,
                      int64_t B, int64_t H, int64_t G, int64_t T, int64_t nt_cap, void* out,
                      void* workspace, size_t workspace_bytes, cudaStream_t st,
                      const float2* stats = nullptr, float stat_scale = 0.f,
                      float2* ml_out = nullptr) {
  int rc = check_decode_shape("value_output", B, H, G, T, nt_cap);
  if (rc) return rc;
  rc = check_codes_aligned("value_output", codes, bits);
  if (rc) return rc;
  if (ld_stats < T) {
    set_error("value_output: ld_stats=%lld < T=%lld", (long long)ld_stats, (long long)T);
    return KVQ_ERR_INVALID;
  }
  const int64_t U = B * H;
  const int64_t nt = (T + kTileTokens - 1) / kTileTokens;
  const int n_splits = value_splits(U, nt, G);
  const size_t part_bytes = align256((size_t)n_splits * U * G * 129 * sizeof(float));
  const size_t base_bytes = value_ws(B, H, G, T);
  const size_t need = stats ? value_scores_ws(B, H, G, T) : base_bytes;
  if (!workspace || workspace_bytes < need) {
    set_error("value_output: workspace too small (%zu < %zu)", workspace_bytes, need);
    return KVQ_ERR_INVALID;
  }
  ValueArgs a{};
  a.codes = codes; a.out_ent = out_ent; a.out_ptr = out_ptr; a.v_scale = v_scale;
  a.v_zero = v_zero; a.ld = ld_stats; a.v_sink = (const __half*)v_sink; a.cb = codebook;
  a.probs = probs; a.B = B; a.H = H; a.G = G; a.T = T; a.nt_cap = nt_cap;
  a.n_splits = n_splits;
  a.stat_scale = stat_scale;
  a.partial = reinterpret_cast<float*>(workspace);
  float* row_max = reinterpret_cast<float*>((char*)workspace + part_bytes);
  unsigned* ml_count = reinterpret_cast<unsigned*>(row_max + B);
  {
    const size_t clear = (size_t)B * sizeof(float) + (stats ? (size_t)U * G * sizeof(unsigned) : 0);
    const cudaError_t me = cudaMemsetAsync(row_max, 0, clear, st);
    if (me != cudaSuccess) {
      set_error("value_output: clearing the row maxima failed: %s", cudaGetErrorString(me));
      return KVQ_ERR_CUDA;
    }
  }
  const unsigned n_chunks = (unsigned)((T + kRowMaxChunk - 1) / kRowMaxChunk);
  if (stats) {
    // one launch: the row maxima and the merge of the key kernel's partials
    const int64_t rows = U * G;
    char* tail = (char*)workspace + base_bytes;
    float2* ml = ml_out ? ml_out : reinterpret_cast<float2*>(tail);
    float2* ml_part = reinterpret_cast<float2*>(tail + align256((size_t)rows * sizeof(float2)));
    a.ml = ml;
    const int n_oct = (int)key_items(T);
    const int n_mc = (int)ml_chunks(T);
    if (B >= 65535) {
      set_error("value_output_scores: batch %lld leaves no grid rows for the softmax merge",
                (long long)B);
      return KVQ_ERR_INVALID;
    }
    const int64_t merge_y = min((rows * n_mc + n_chunks - 1) / n_chunks, (int64_t)65535 - B);
    value_prep_kernel<<<dim3(n_chunks, (unsigned)(B + merge_y)), 256, 0, st>>>(
        v_scale, T, ld_stats, row_max, B, stats, n_oct, rows, n_mc, ml_part, ml_count, ml);
  } else {
    row_max_kernel<<<dim3(n_chunks, (unsigned)B), 256, 0, st>>>(v_scale, T, ld_stats, row_max);
  }
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


inline size_t stats_ws(int64_t rows, int64_t T) {
  return align256((size_t)(rows > 0 ? rows : 0) * key_items(T > 0 ? T : 0) * sizeof(float2));
}

// Workspace of decode_attention: [scores][probs][softmax partials][value partials][key stats].
struct DecodeWs {
  size_t scores, probs, soft, value, stats, total;
};
inline DecodeWs decode_ws(int64_t B, int64_t H, int64_t G, int64_t T) {
  DecodeWs w;
  const int64_t rows = B * H * G;
  w.scores = align256((size_t)rows * T * sizeof(float));
  w.probs = w.scores;
  w.soft = softmax_ws(rows, T);
  w.value = value_scores_ws(B, H, G, T);  // room for either variant
  w.stats = stats_ws(rows, T);
  w.total = w.scores + w.probs + w.soft + w.value + w.stats;
  return w;
}

}  // namespace kvq

namespace kvq {
static int key_impl(const uint8_t* codes, const uint32_t* out_ent, const int32_t* out_ptr,
                    const float* k_scale, const float* k_zero, const void* k_sink,
                    const float* codebook, int bits, const void* q, const float* inv_freq,
                    int64_t B, int64_t n_heads, int64_t group, int64_t T, int64_t nt_cap,
                    float* scores, float2* stats, float stat_scale, cudaStream_t st,
                    int64_t pos0 = 0) {
  int rc = check_decode_shape("key_scores", B, n_heads, group, T, nt_cap);
  if (rc) return rc;
  rc = check_codes_aligned("key_scores", codes, bits);
  if (rc) return rc;
  if (pos0 < 0 || pos0 + T > (1LL << 24)) {  // positions are exact fp32 integers up to 2^24
    set_error("key_scores: positions [%lld, %lld) outside [0, 2^24]", (long long)pos0,
              (long long)(pos0 + T));
    return KVQ_ERR_INVALID;
  }
  KeyArgs a{};
  a.codes = codes; a.out_ent = out_ent; a.out_ptr = out_ptr; a.k_scale = k_scale;
  a.k_zero = k_zero; a.k_sink = (const __half*)k_sink; a.cb = codebook; a.q = (const __half*)q;
  a.inv_freq = inv_freq; a.B = B; a.H = n_heads; a.G = group; a.T = T; a.nt_cap = nt_cap;
  a.scores = scores;
  a.stats = stats;
  a.stat_scale = stat_scale;
  a.pos0 = pos0;
  switch (group) {
    case 1: return dispatch_key_bits<1>(bits, a, st);
    case 2: return dispatch_key_bits<2>(bits, a, st);
    case 4: return dispatch_key_bits<4>(bits, a, st);
    case 8: return dispatch_key_bits<8>(bits, a, st);
  }
  return KVQ_ERR_UNSUPPORTED;
}
}  // namespace kvq

extern "C" int kvq_set_decode_kernels(int key_kernel, int value_kernel) {
  if (key_kernel < -1 || key_kernel > 1 || value_kernel < -1 || value_kernel > 1) {
    kvq::set_error("kvq_set_decode_kernels: kernels are -1 (keep), 0 (mma.sync), 1 (tcgen05)");
    return KVQ_ERR_INVALID;
  }
  if (key_kernel >= 0) kvq::g_key_kernel().store(key_kernel);
  if (value_kernel >= 0) kvq::g_value_kernel().store(value_kernel);
  return KVQ_OK;
}

extern "C" int kvq_decode_kernels(void) {
  return kvq::g_key_kernel().load() | (kvq::g_value_kernel().load() << 1);
}

extern "C" int kvq_key_scores(const uint8_t* codes, const uint32_t* out_ent,
                              const int32_t* out_ptr, const float* k_scale, const float* k_zero,
                              const void* k_sink, const float* codebook, int bits, const void* q,
                              const float* inv_freq, int64_t B, int64_t n_heads, int64_t group,
                              int64_t T, int64_t nt_cap, float* scores, void* stream) {
  kvq::clear_error();
  return kvq::key_impl(codes, out_ent, out_ptr, k_scale, k_zero, k_sink, codebook, bits, q,
                       inv_freq, B, n_heads, group, T, nt_cap, scores, nullptr, 0.f,
                       kvq::as_stream(stream));
}

extern "C" size_t kvq_key_stats_size(int64_t rows, int64_t T) {
  if (rows <= 0 || T <= 0) return 0;
  return (size_t)rows * kvq::key_items(T) * sizeof(float2);
}

extern "C" int kvq_key_scores_stats(const uint8_t* codes, const uint32_t* out_ent,
                                    const int32_t* out_ptr, const float* k_scale,
                                    const float* k_zero, const void* k_sink,
                                    const float* codebook, int bits, const void* q,
                                    const float* inv_freq, int64_t B, int64_t n_heads,
                                    int64_t group, int64_t T, int64_t nt_cap, float* scores,
                                    float scale, void* stats, void* stream) {
  kvq::clear_error();
  if (!stats) {
    kvq::set_error("key_scores_stats: stats is NULL");
    return KVQ_ERR_INVALID;
  }
  return kvq::key_impl(codes, out_ent, out_ptr, k_scale, k_zero, k_sink, codebook, bits, q,
                       inv_freq, B, n_heads, group, T, nt_cap, scores,
                       reinterpret_cast<float2*>(stats), scale, kvq::as_stream(stream));
}

extern "C" int kvq_key_scores_stats_at(const uint8_t* codes, const uint32_t* out_ent,
                                       const int32_t* out_ptr, const float* k_scale,
                                       const float* k_zero, const void* k_sink,
                                       const float* codebook, int bits, const void* q,
                                       const float* inv_freq, int64_t B, int64_t n_heads,
                                       int64_t group, int64_t T, int64_t nt_cap, int64_t pos0,
                                       float* scores, float scale, void* stats, void* stream) {
  kvq::clear_error();
  if (!stats) {
    kvq::set_error("key_scores_stats_at: stats is NULL");
    return KVQ_ERR_INVALID;
  }
  if (k_sink && pos0 != 0) {  // the sink is position 0, scored without rotation
    kvq::set_error("key_scores_stats_at: a sink token needs pos0 == 0 (got %lld)",
                   (long long)pos0);
    return KVQ_ERR_INVALID;
  }
  return kvq::key_impl(codes, out_ent, out_ptr, k_scale, k_zero, k_sink, codebook, bits, q,
                       inv_freq, B, n_heads, group, T, nt_cap, scores,
                       reinterpret_cast<float2*>(stats), scale, kvq::as_stream(stream), pos0);
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

extern "C" size_t kvq_value_output_scores_workspace(int64_t B, int64_t n_heads, int64_t group,
                                                    int64_t T) {
  return kvq::value_scores_ws(B, n_heads, group, T);
}

extern "C" int kvq_value_output_scores(const uint8_t* codes, const uint32_t* out_ent,
                                       const int32_t* out_ptr, const float* v_scale,
                                       const float* v_zero, int64_t ld_stats, const void* v_sink,
                                       const float* codebook, int bits, const float* scores,
                                       const void* stats, float scale, int64_t B,
                                       int64_t n_heads, int64_t group, int64_t T, int64_t nt_cap,
                                       void* out, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  kvq::clear_error();
  if (!stats) {
    kvq::set_error("value_output_scores: stats is NULL");
    return KVQ_ERR_INVALID;
  }
  return kvq::value_impl(codes, out_ent, out_ptr, v_scale, v_zero, ld_stats, v_sink, codebook,
                         bits, scores, B, n_heads, group, T, nt_cap, out, workspace,
                         workspace_bytes, kvq::as_stream(stream),
                         reinterpret_cast<const float2*>(stats), scale);
}

extern "C" int kvq_value_output_scores_ml(const uint8_t* codes, const uint32_t* out_ent,
                                          const int32_t* out_ptr, const float* v_scale,
                                          const float* v_zero, int64_t ld_stats,
                                          const void* v_sink, const float* codebook, int bits,
                                          const float* scores, const void* stats, float scale,
                                          int64_t B, int64_t n_heads, int64_t group, int64_t T,
                                          int64_t nt_cap, void* out, float* ml_out,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  kvq::clear_error();
  if (!stats || !ml_out) {
    kvq::set_error("value_output_scores_ml: stats and ml_out are required");
    return KVQ_ERR_INVALID;
  }
  return kvq::value_impl(codes, out_ent, out_ptr, v_scale, v_zero, ld_stats, v_sink, codebook,
                         bits, scores, B, n_heads, group, T, nt_cap, out, workspace,
                         workspace_bytes, kvq::as_stream(stream),
                         reinterpret_cast<const float2*>(stats), scale,
                         reinterpret_cast<float2*>(ml_out));
}

extern "C" int kvq_merge_shards(const void* o_shards, const float* ml_shards, int64_t n_shards,
                                int64_t rows, void* out, void* stream) {
  kvq::clear_error();
  if (n_shards < 1 || rows < 0 || rows > (1LL << 31) - 1 || !o_shards || !ml_shards || !out) {
    kvq::set_error("merge_shards: invalid arguments (n_shards=%lld, rows=%lld)",
                   (long long)n_shards, (long long)rows);
    return KVQ_ERR_INVALID;
  }
  if (rows == 0) return KVQ_OK;
  kvq::merge_shards_kernel<<<(unsigned)rows, kvq::kHeadDim, 0, kvq::as_stream(stream)>>>(
      (const __half*)o_shards, reinterpret_cast<const float2*>(ml_shards), n_shards, rows,
      (__half*)out);
  return kvq::check_launch("merge_shards");
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
  float2* stats = reinterpret_cast<float2*>(ws + w.scores + w.probs + w.soft + w.value);
  const float scale = 0.08838834764831845f;  // 1 / sqrt(128)
  cudaStream_t st = as_stream(stream);
  if (!probs_out) {
    // fused softmax: the key kernel leaves per-item partials, the value kernel
    // turns the raw scores into probabilities itself
    rc = key_impl(k_codes, k_out_ent, k_out_ptr, k_scale, k_zero, k_sink, k_codebook, bits, q,
                  inv_freq, B, n_heads, group, T, nt_cap, scores, stats, scale, st);
    if (rc) return rc;
    return value_impl(v_codes, v_out_ent, v_out_ptr, v_scale, v_zero, ld_stats, v_sink,
                      v_codebook, bits, scores, B, n_heads, group, T, nt_cap, out, val, w.value,
                      st, stats, scale);
  }
  rc = key_impl(k_codes, k_out_ent, k_out_ptr, k_scale, k_zero, k_sink, k_codebook, bits, q,
                inv_freq, B, n_heads, group, T, nt_cap, scores, nullptr, 0.f, st);
  if (rc) return rc;
  rc = softmax_impl(scores, B * n_heads * group, T, scale, probs, soft, w.soft, st);
  if (rc) return rc;
  return value_impl(v_codes, v_out_ent, v_out_ptr, v_scale, v_zero, ld_stats, v_sink, v_codebook,
                    bits, probs, B, n_heads, group, T, nt_cap, out, val, w.value, st);
}
