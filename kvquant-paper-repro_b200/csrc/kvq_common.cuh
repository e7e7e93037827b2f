// Shared definitions for the kvquant_b200 sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/kvquant_b200.h"

namespace kvq {

constexpr int kTileTokens = 32;   // tokens per code tile
constexpr int kHeadDim = 128;     // channels per head
constexpr int kPairs = 64;        // RoPE rotate-half pairs per head

__host__ __device__ inline int tile_bytes(int bits) { return kTileTokens * kHeadDim * bits / 8; }

// Thread-local error message of the last failed entry point.
void set_error(const char* fmt, ...);
void clear_error();

// Device-side sticky status word (set by kernels that skip an invalid access).
// Single definition: the library is built as one translation unit (kvq_lib.cu).
__device__ int g_status = 0;
enum StatusBits : int { kStatusBadIndex = 1 };

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Returns KVQ_OK, or KVQ_ERR_CUDA with the message recorded.
int check_launch(const char* what);

// Outlier count k = max(1, min(int(n * ratio), n)) (kvquant/quant/dense_sparse.py:22-23),
// with Python's float semantics (IEEE double product, truncation toward 0).
inline int64_t outlier_count(int64_t n, double ratio) {
  if (n <= 0) return 0;
  int64_t k = (int64_t)(double(n) * ratio);
  if (k > n) k = n;
  if (k < 1) k = 1;
  return k;
}

// Normalization n = (x - zero) / (scale + 1e-8) with IEEE fp32 rounding of every
// step (kvquant/quant/kv_quantizer.py:82,110); never contracted into an FMA.
__device__ __forceinline__ float normalize(float x, float zero, float scale) {
  return __fdiv_rn(__fsub_rn(x, zero), __fadd_rn(scale, 1e-8f));
}

// The same normalization for many x sharing (zero, scale), with the division
// done from the correctly rounded reciprocal y = RN(1/b), b = scale + 1e-8:
// q0 = RN(a y) is within 1.5 ulp of a/b, one correction q1 = RN(q0 + RN(a -
// b q0) y) makes it faithful, and by Markstein's theorem (a faithful quotient
// q and y within half an ulp of 1/b give RN(q + (a - b q) y) = RN(a/b), the
// remainder a - b q being exact in an FMA) a second correction rounds it
// correctly. Five FP instructions instead of a division. The theorem needs
// every quantity to stay normal, which holds for fp16 inputs x when b is in
// [2^-60, 2^30] and zero is 0 or of magnitude in [2^-60, 2^60] (then a =
// x - zero is 0 or at least 2^-84 in magnitude, and a/b is 0 or between
// 2^-114 and 2^77); `fast` is false otherwise and for infinite or NaN a,
// where the IEEE division runs.
struct Normalizer {
  float z, b, y;
  bool fast;
  __device__ __forceinline__ void init(float zero, float scale) {
    z = zero;
    b = __fadd_rn(scale, 1e-8f);
    y = __frcp_rn(b);
    const float az = fabsf(zero);
    fast = (az == 0.f || (az >= 0x1p-60f && az <= 0x1p60f)) && b >= 0x1p-60f && b <= 0x1p30f;
  }
  // a / b for a = x - zero, valid when `fast` holds and x is finite
  __device__ __forceinline__ float quot(float x) const {
    const float a = __fsub_rn(x, z);
    float q = __fmul_rn(a, y);
    float r = __fmaf_rn(-q, b, a);
    q = __fmaf_rn(r, y, q);
    r = __fmaf_rn(-q, b, a);
    q = __fmaf_rn(r, y, q);
    return a == 0.f ? a : q;  // the corrections turn -0 into +0; IEEE keeps the sign
  }
  __device__ __forceinline__ float operator()(float x) const {
    if (!fast || !(fabsf(x) < INFINITY)) return __fdiv_rn(__fsub_rn(x, z), b);
    return quot(x);
  }
};

// True when all eight fp16 values of a 16-byte chunk are finite.
__device__ __forceinline__ bool finite8(const uint4& v) {
  auto ok = [](uint32_t w) {
    return (w & 0x7C00u) != 0x7C00u && (w & 0x7C000000u) != 0x7C000000u;
  };
  return ok(v.x) && ok(v.y) && ok(v.z) && ok(v.w);
}

// First-minimum nearest centroid (kvquant/kernels/csrc/kvquant_ops.cu:141-148).
__device__ __forceinline__ int nearest_centroid(float v, const float* cb, int n) {
  float best_d = fabsf(__fsub_rn(v, cb[0]));
  int best = 0;
  for (int k = 1; k < n; ++k) {
    float d = fabsf(__fsub_rn(v, cb[k]));
    if (d < best_d) { best_d = d; best = k; }
  }
  return best;
}

// The same rule in O(log n) over the codebook sorted ascending (sv, with the
// original indices si; equal values keep their original order). fl(v - c) is
// non-increasing in c, so over the sorted codebook the rounded distances
// |fl(v - c)| fall up to the last entry <= v and rise after it; the entries at
// the minimal distance therefore form one contiguous run around that boundary,
// and the first minimum of the original order is the lowest original index in
// the run. n is a power of two <= 16.
__device__ __forceinline__ int nearest_centroid_sorted(float v, const float* sv, const uint8_t* si,
                                                       int n) {
  int j = 0;  // number of entries <= v: binary search, then the last step
#pragma unroll
  for (int step = 8; step >= 1; step >>= 1)
    if (step < n && sv[j + step - 1] <= v) j += step;
  if (sv[j] <= v) ++j;  // here j <= n - 1
  float m = INFINITY;
  if (j > 0) m = fabsf(__fsub_rn(v, sv[j - 1]));
  if (j < n) m = fminf(m, fabsf(__fsub_rn(v, sv[j])));
  int best = 255;
  for (int k = j - 1; k >= 0 && fabsf(__fsub_rn(v, sv[k])) == m; --k) best = min(best, (int)si[k]);
  for (int k = j; k < n && fabsf(__fsub_rn(v, sv[k])) == m; ++k) best = min(best, (int)si[k]);
  return best;
}

// Sorts a codebook of n <= 16 entries ascending (stable) with its original
// indices; one thread.
__device__ __forceinline__ void sort_codebook(const float* cb, int n, float* sv, uint8_t* si) {
  for (int k = 0; k < n; ++k) {
    const float x = cb[k];
    int p = k;
    while (p > 0 && sv[p - 1] > x) {
      sv[p] = sv[p - 1];
      si[p] = si[p - 1];
      --p;
    }
    sv[p] = x;
    si[p] = (uint8_t)k;
  }
}

// Fake-quant dequantization (q + o) * s + z with the reference's fp32 op order
// (kvquant/quant/kv_quantizer.py:89,117): add, multiply, add, each rounded.
__device__ __forceinline__ float dequant_ref(float cbq, float o, float s, float z) {
  return __fadd_rn(__fmul_rn(__fadd_rn(cbq, o), s), z);
}

// Mixed-precision FMA: fp16 x fp16 (exact product) + fp32 -> fp32 (sm_100 `fma.rn.f32.f16`).
__device__ __forceinline__ float fma_h(uint16_t a, uint16_t b, float c) {
  float r;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(r) : "h"(a), "h"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t lo16(uint32_t w) { return w & 0xffffu; }
__device__ __forceinline__ uint32_t hi16(uint32_t w) { return w >> 16; }

// Splits a 32-bit register into its two 16-bit halves as a register-level
// view (no arithmetic), so half-operand instructions can read them in place.
__device__ __forceinline__ void unpack16(uint32_t w, uint16_t& lo, uint16_t& hi) {
  asm("mov.b32 {%0, %1}, %2;" : "=h"(lo), "=h"(hi) : "r"(w));
}

__device__ __forceinline__ uint32_t half2_bits(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Extracts the 2*bits-wide code pair m from a slab held in registers
// (little-endian bit stream; pair m at bits [2*bits*m, 2*bits*(m+1))).
template <int BITS>
__device__ __forceinline__ uint32_t slab_pair(const uint32_t* w, int m) {
  constexpr int W = 2 * BITS;
  const int bit = W * m;
  const int wi = bit >> 5, sh = bit & 31;
  uint32_t lo = w[wi] >> sh;
  if (sh + W > 32) lo |= w[wi + 1] << (32 - sh);
  return lo & ((1u << W) - 1u);
}

}  // namespace kvq
