// The reference's four ops (kvquant/kernels/csrc/kvquant_ops.cu:265-270) as
// sm_100a kernels behind the C ABI. Same argument meaning and results; the
// hidden dtype/contiguity copies of the reference's host wrappers are the
// Python binding's job, so these entry points take dense buffers only.
#pragma once
#include "kvq_common.cuh"

namespace kvq {

// ---------------------------------------------------------------------------
// RoPE (rotate-half), kvquant_ops.cu:27-55. One thread per (row, 2 pairs):
// rows are (b,h,s); pair index p pairs channel p with p + D/2.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rope_apply_kernel(
    const __half* __restrict__ x, const float* __restrict__ cos_tab,
    const float* __restrict__ sin_tab, __half* __restrict__ out, int64_t rows, int S, int D,
    int64_t pos_offset) {
  const int half_d = D >> 1;
  const int64_t total = rows * half_d;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(idx % half_d);
    const int64_t row = idx / half_d;
    const int s = (int)(row % S);
    const int64_t pos = s + pos_offset;
    const float c = __ldg(cos_tab + pos * half_d + p);
    const float sn = __ldg(sin_tab + pos * half_d + p);
    const __half* xr = x + row * D;
    const float x1 = __half2float(xr[p]);
    const float x2 = __half2float(xr[p + half_d]);
    __half* orow = out + row * D;
    orow[p] = __float2half_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn)));
    orow[p + half_d] = __float2half_rn(__fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, c)));
  }
}

// ---------------------------------------------------------------------------
// LUT matvec, kvquant_ops.cu:62-100: one warp per row, fp32 accumulation,
// 16-byte code loads when the row is 16-byte aligned.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) lut_matvec_kernel(
    const uint8_t* __restrict__ qmat, const __half* __restrict__ lut, int lut_size,
    const __half* __restrict__ scale, const __half* __restrict__ zero,
    const __half* __restrict__ vec, __half* __restrict__ out, int64_t N, int D, int per_channel,
    int vec16) {
  __shared__ float s_lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    s_lut[i] = i < lut_size ? __half2float(lut[i]) : 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < N;
       row += warps) {
    const uint8_t* rp = qmat + row * D;
    float acc = 0.f;
    const float rs = per_channel ? 0.f : __half2float(scale[row]);
    const float rz = per_channel ? 0.f : __half2float(zero[row]);
    auto term = [&](int j, uint32_t code) {
      // Table entries at or beyond lut_size read as 0 (the reference leaves them
      // uninitialized); every uint8 code indexes inside the 256-entry table.
      const float l = s_lut[code];
      const float sc = per_channel ? __half2float(scale[j]) : rs;
      const float zc = per_channel ? __half2float(zero[j]) : rz;
      acc = fmaf(fmaf(l, sc, zc), __half2float(vec[j]), acc);
    };
    if (vec16) {
      for (int j0 = lane * 16; j0 < D; j0 += 32 * 16) {
        const uint4 w = *reinterpret_cast<const uint4*>(rp + j0);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int b = 0; b < 16; ++b) term(j0 + b, (ws[b >> 2] >> (8 * (b & 3))) & 0xffu);
      }
    } else {
      for (int j = lane; j < D; j += 32) term(j, rp[j]);
    }
    acc = warp_sum(acc);
    if (lane == 0) out[row] = __float2half_rn(acc);
  }
}

// ---------------------------------------------------------------------------
// CSR sparse matvec, kvquant_ops.cu:106-127: one warp per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) sparse_matvec_csr_kernel(
    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
    const __half* __restrict__ val, const __half* __restrict__ vec, __half* __restrict__ out,
    int64_t R, int64_t nnz, int64_t vec_len) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < R;
       r += warps) {
    int64_t s = row_ptr[r], e = row_ptr[r + 1];
    float acc = 0.f;
    if (s < 0 || e > nnz || s > e) {
      if (lane == 0) atomicOr(&g_status, kStatusBadIndex);
    } else {
      for (int64_t k = s + lane; k < e; k += 32) {
        const int32_t c = col[k];
        if (c < 0 || c >= vec_len) {
          atomicOr(&g_status, kStatusBadIndex);
          continue;
        }
        acc = fmaf(__half2float(val[k]), __half2float(vec[c]), acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) out[r] = __float2half_rn(acc);
  }
}

// ---------------------------------------------------------------------------
// Nearest-centroid lookup, kvquant_ops.cu:132-151 (first minimum wins).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) lut_lookup_kernel(
    const float* __restrict__ x, const float* __restrict__ cb, int lut_size,
    int64_t* __restrict__ idx_out, float* __restrict__ dq_out, int64_t N) {
  __shared__ float s_cb[256];
  const bool in_smem = lut_size <= 256;
  if (in_smem)
    for (int i = threadIdx.x; i < lut_size; i += blockDim.x) s_cb[i] = cb[i];
  __syncthreads();
  const float* c = in_smem ? s_cb : cb;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int best = nearest_centroid(x[i], c, lut_size);
    idx_out[i] = best;
    dq_out[i] = c[best];
  }
}

inline int grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  const int64_t cap = 148LL * 32;  // grid-stride loops beyond this
  return (int)(g < cap ? g : cap);
}

}  // namespace kvq

using namespace kvq;

extern "C" int kvq_rope_apply(const void* x, const float* cos_tab, const float* sin_tab,
                              void* out, int64_t B, int64_t H, int64_t S, int64_t D,
                              int64_t pos_offset, int64_t s_total, void* stream) {
  clear_error();
  if (B < 0 || H < 0 || S < 0 || D <= 0 || (D & 1) || pos_offset < 0 ||
      pos_offset + S > s_total) {
    set_error("rope_apply: invalid shape B=%lld H=%lld S=%lld D=%lld pos_offset=%lld "
              "s_total=%lld (need even D and pos_offset+S <= s_total)",
              (long long)B, (long long)H, (long long)S, (long long)D, (long long)pos_offset,
              (long long)s_total);
    return KVQ_ERR_INVALID;
  }
  const int64_t rows = B * H * S;
  if (rows == 0) return KVQ_OK;
  if (!x || !cos_tab || !sin_tab || !out) {
    set_error("rope_apply: null pointer");
    return KVQ_ERR_INVALID;
  }
  rope_apply_kernel<<<grid_for(rows * (D / 2), 256), 256, 0, as_stream(stream)>>>(
      (const __half*)x, cos_tab, sin_tab, (__half*)out, rows, (int)S, (int)D, pos_offset);
  return check_launch("rope_apply");
}

extern "C" int kvq_lut_matvec(const uint8_t* qmat, const void* lut, int64_t lut_size,
                              const void* scale, const void* zero, const void* vec, void* out,
                              int64_t N, int64_t D, int per_channel, void* stream) {
  clear_error();
  if (lut_size < 1 || lut_size > 256) {
    set_error("lut_matvec: lut_size too large (%lld, need 1..256)", (long long)lut_size);
    return KVQ_ERR_INVALID;
  }
  if (N < 0 || D < 0) {
    set_error("lut_matvec: invalid shape N=%lld D=%lld", (long long)N, (long long)D);
    return KVQ_ERR_INVALID;
  }
  if (N == 0) return KVQ_OK;
  const int vec16 = (D % 16 == 0) && ((uintptr_t)qmat % 16 == 0);
  lut_matvec_kernel<<<grid_for(N, 8), 256, 0, as_stream(stream)>>>(
      qmat, (const __half*)lut, (int)lut_size, (const __half*)scale, (const __half*)zero,
      (const __half*)vec, (__half*)out, N, (int)D, per_channel, vec16);
  return check_launch("lut_matvec");
}

extern "C" int kvq_sparse_matvec_csr(const int32_t* row_ptr, const int32_t* col_idx,
                                     const void* values, const void* vec, void* out, int64_t R,
                                     int64_t nnz, int64_t vec_len, void* stream) {
  clear_error();
  if (R < 0 || nnz < 0 || vec_len < 0) {
    set_error("sparse_matvec_csr: invalid sizes R=%lld nnz=%lld", (long long)R,
              (long long)nnz);
    return KVQ_ERR_INVALID;
  }
  if (R == 0) return KVQ_OK;
  sparse_matvec_csr_kernel<<<grid_for(R, 8), 256, 0, as_stream(stream)>>>(
      row_ptr, col_idx, (const __half*)values, (const __half*)vec, (__half*)out, R, nnz,
      vec_len);
  return check_launch("sparse_matvec_csr");
}

extern "C" int kvq_lut_lookup(const float* x, const float* codebook, int64_t lut_size,
                              int64_t* idx_out, float* dq_out, int64_t N, void* stream) {
  clear_error();
  if (lut_size < 1 || lut_size > (1 << 24) || N < 0) {
    set_error("lut_lookup: invalid lut_size=%lld N=%lld", (long long)lut_size, (long long)N);
    return KVQ_ERR_INVALID;
  }
  if (N == 0) return KVQ_OK;
  lut_lookup_kernel<<<grid_for(N, 256), 256, 0, as_stream(stream)>>>(
      x, codebook, (int)lut_size, idx_out, dq_out, N);
  return check_launch("lut_lookup");
}

// The reference's normalization n = (x - zero) / (scale + 1e-8) of quantize_k /
// quantize_v (kvquant/quant/kv_quantizer.py:82,104) in the form the quantize
// kernels compute it (Normalizer: reciprocal, two corrections, IEEE division
// where its guards fail). x fp16 [rows, cols]; zero / scale fp32 per column
// (per_channel, keys) or per row (values); out fp32.
namespace kvq {
__global__ void normalize_kernel(const __half* __restrict__ x, int64_t rows, int64_t cols,
                                 const float* __restrict__ zero, const float* __restrict__ scale,
                                 int per_channel, float* __restrict__ out) {
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = per_channel ? i % cols : i / cols;
    Normalizer nz;
    nz.init(zero[k], scale[k]);
    out[i] = nz(__half2float(x[i]));
  }
}
}  // namespace kvq

extern "C" int kvq_normalize(const void* x, int64_t rows, int64_t cols, const float* zero,
                             const float* scale, int per_channel, float* out, void* stream) {
  using namespace kvq;
  clear_error();
  if (rows < 0 || cols < 0) {
    set_error("normalize: invalid shape rows=%lld cols=%lld", (long long)rows, (long long)cols);
    return KVQ_ERR_INVALID;
  }
  if (rows == 0 || cols == 0) return KVQ_OK;
  normalize_kernel<<<grid_for(rows * cols, 256), 256, 0, as_stream(stream)>>>(
      (const __half*)x, rows, cols, zero, scale, per_channel, out);
  return check_launch("normalize");
}
