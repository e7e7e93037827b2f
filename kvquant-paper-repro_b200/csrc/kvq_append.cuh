// Decode-time append: quantizes new tokens into an existing packed cache at
// positions [T_old, T_old + S_new) without touching the rest of it.
//
// Values follow KVQuantizer.quantize_v token by token (kvquant/quant/
// kv_quantizer.py:96-122): per-token scale/zero over all C channels and the
// top-k outliers over C, exactly as a one-token call of the reference does.
// Keys use per-channel outlier thresholds on |n| (the calibrated-threshold
// scheme of the KVQuant paper, section 3.4): |n| >= thr[c] is an outlier. With
// thr = 0 every channel is an outlier, which is what the reference's
// quantize_k does with a one-token block (k = max(1, int(1 * r)) = 1 per
// channel, dense_sparse.py:22-23).
//
// The cache must have room: a spare tile after the last appended token, and
// per-unit outlier segments (unit u owns entries [u * ent_stride,
// (u + 1) * ent_stride)), the layout that kvquant.kernels.make_appendable
// builds. The decode kernels read it unchanged: they only look at row
// pointers up to the end of the last filled tile of each unit.
#pragma once
#include "kvq_quantize.cuh"

namespace kvq {

struct AppendArgs {
  const __half* x;  // new tokens [B, S_new, C_full]
  int64_t B, S_new, C_full, h0, H;
  int64_t T_old;            // tokens already in the cache (>= 1)
  const float* k_scale;     // keys: [n_heads*128] (the cache's local channels)
  const float* k_zero;
  const float* k_thr;       // keys: [n_heads*128] outlier thresholds on |n|
  const float* v_scale;     // values: [B, ld] per-token stats (new positions filled)
  const float* v_zero;
  int64_t ld_stats;
  const Select* sel;        // values: [B * S_new] per-token selections
  bool outliers;
  const float* cb;
  int bits;
  uint8_t* codes;
  int64_t nt_cap;
  int32_t* out_ptr;
  uint32_t* out_ent;
  int64_t ent_stride;       // entries per unit segment
  int32_t* status;          // bit 0: a unit's segment had no room (nothing written for it)
};

// Token / channel of the two codes of slot q in lane (g, cc)'s slab of block blk
// (the fragment-native order of the decode kernels; the same map the emit
// kernel packs with).
template <int KIND>
__device__ __forceinline__ void slot_map(int q, int blk, int g, int cc, int& ta, int& ca, int& tb,
                                         int& cb2) {
  if (KIND == 0) {  // keys: token 16*blk + g + 8*(q&1), RoPE pair 4*(q>>1) + cc
    ta = tb = 16 * blk + g + 8 * (q & 1);
    ca = 4 * (q >> 1) + cc;
    cb2 = ca + 64;
  } else {          // values: channel 16*(q>>2) + g + 8*(q&1), tokens (t, t+1)
    ca = cb2 = 16 * (q >> 2) + g + 8 * (q & 1);
    ta = 16 * blk + 2 * cc + 8 * ((q >> 1) & 1);
    tb = ta + 1;
  }
}

// One CTA of 128 threads (thread = channel of the head) per (head, b) unit. It
// first counts the unit's new outliers and gives up (status bit) if its
// segment cannot take them; otherwise it walks the touched tiles in order:
// unpacks the old tokens' codes of the tile, quantizes the new tokens,
// appends their outlier entries in (token, channel) order behind the unit's
// last entry, moves the tile's two row pointers and rewrites the tile's slabs.
template <int KIND, int BITS>
__global__ void __launch_bounds__(128) append_kernel(AppendArgs a) {
  __shared__ __align__(16) __half xs[kTileTokens][kHeadDim];
  __shared__ int32_t cnt[kTileTokens][8];
  __shared__ float s_cb[16], s_cbs[16];
  __shared__ uint8_t s_cbi[16];
  __shared__ uint8_t s_code[kTileTokens][kHeadDim];
  __shared__ float s_vs[kTileTokens], s_vz[kTileTokens];
  __shared__ Select s_rs[kTileTokens];
  __shared__ int32_t s_red[4];
  __shared__ int32_t s_n0, s_tot;
  const int64_t h = blockIdx.x, b = blockIdx.y;
  const int c = threadIdx.x, lane = c & 31, w = c >> 5;
  const int64_t unit = b * a.H + h;
  constexpr int ncb = 1 << BITS;
  const int64_t cfull = (a.h0 + h) * kHeadDim + c;
  const int64_t T_new = a.T_old + a.S_new;
  const int64_t urow = unit * 2 * a.nt_cap;  // first CSR row of the unit
  if (c == 0) {
    for (int k = 0; k < ncb; ++k) s_cb[k] = a.cb[k];
    sort_codebook(s_cb, ncb, s_cbs, s_cbi);
  }
  float kz = 0.f, ks = 0.f, kt = 0.f;
  if (KIND == 0) {
    const int64_t cl = h * kHeadDim + c;
    kz = a.k_zero[cl];
    ks = a.k_scale[cl];
    kt = a.outliers ? a.k_thr[cl] : 0.f;
  }
  // Pass 1: this unit's new outliers.
  int32_t mine = 0;
  if (a.outliers) {
    for (int64_t t = a.T_old; t < T_new; ++t) {
      const int64_t r = b * a.S_new + (t - a.T_old);
      const float xv = __half2float(a.x[r * a.C_full + cfull]);
      bool out;
      if (KIND == 0) {
        out = fabsf(normalize(xv, kz, ks)) >= kt;
      } else {
        const float n = normalize(xv, a.v_zero[b * a.ld_stats + t], a.v_scale[b * a.ld_stats + t]);
        out = selected(abs_bits(n), (int32_t)cfull, a.sel[r]);
      }
      mine += out ? 1 : 0;
    }
  }
  mine = __reduce_add_sync(0xffffffffu, mine);
  if (lane == 0) s_red[w] = mine;
  __syncthreads();
  const int64_t total = (int64_t)s_red[0] + s_red[1] + s_red[2] + s_red[3];
  const int64_t tl = a.T_old - 1;  // last token already cached
  int64_t end = a.out_ptr[urow + 2 * (tl / kTileTokens) + (tl % kTileTokens) / 16 + 1];
  if (end < unit * a.ent_stride || end + total > (unit + 1) * a.ent_stride) {
    if (c == 0) atomicOr(a.status, 1);
    return;  // the whole CTA leaves here: the decision is uniform
  }

  for (int64_t tile = a.T_old / kTileTokens; tile <= (T_new - 1) / kTileTokens; ++tile) {
    const int64_t t0 = tile * kTileTokens;
    uint8_t* tile_base = a.codes + (unit * a.nt_cap + tile) * (int64_t)(kTileTokens * kHeadDim * BITS / 8);
    for (int k = c; k < kTileTokens * kHeadDim; k += 128) (&s_code[0][0])[k] = 0;
    __syncthreads();
    // Old tokens' codes of the tile: threads 0..63 unpack slab (block, lane).
    if (t0 < a.T_old && c < 64) {
      const int blk = c >> 5, g = lane >> 2, cc = lane & 3;
      const uint8_t* bb = tile_base + blk * (256 * BITS);
      uint32_t slab[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      const uint4 v0 = *reinterpret_cast<const uint4*>(bb + lane * 16);
      slab[0] = v0.x; slab[1] = v0.y; slab[2] = v0.z; slab[3] = v0.w;
      if (BITS == 4) {
        const uint4 v1 = *reinterpret_cast<const uint4*>(bb + 512 + lane * 16);
        slab[4] = v1.x; slab[5] = v1.y; slab[6] = v1.z; slab[7] = v1.w;
      } else if (BITS == 3) {
        const uint2 v1 = *reinterpret_cast<const uint2*>(bb + 512 + lane * 8);
        slab[4] = v1.x; slab[5] = v1.y;
      }
      constexpr uint32_t cmask = (1u << BITS) - 1u;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        int ta, ca, tb, cb2;
        slot_map<KIND>(q, blk, g, cc, ta, ca, tb, cb2);
        const uint32_t pair = slab_pair<BITS>(slab, q);
        if (t0 + ta < a.T_old) s_code[ta][ca] = (uint8_t)(pair & cmask);
        if (t0 + tb < a.T_old) s_code[tb][cb2] = (uint8_t)(pair >> BITS);
      }
    }
    // New tokens of the tile, staged with coalesced 16-byte loads.
    for (int k = c; k < kTileTokens * (kHeadDim / 8); k += 128) {
      const int i = k >> 4, ch8 = (k & 15) * 8;
      const int64_t t = t0 + i;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (t >= a.T_old && t < T_new)
        v = *reinterpret_cast<const uint4*>(a.x + (b * a.S_new + (t - a.T_old)) * a.C_full +
                                            (a.h0 + h) * kHeadDim + ch8);
      *reinterpret_cast<uint4*>(&xs[i][ch8]) = v;
    }
    if (KIND == 1 && c < kTileTokens) {
      const int64_t t = t0 + c;
      const bool live = t >= a.T_old && t < T_new;
      s_vs[c] = live ? a.v_scale[b * a.ld_stats + t] : 0.f;
      s_vz[c] = live ? a.v_zero[b * a.ld_stats + t] : 0.f;
      if (live && a.outliers) s_rs[c] = a.sel[b * a.S_new + (t - a.T_old)];
    }
    __syncthreads();

    uint32_t omask = 0;
    float nval[kTileTokens];
#pragma unroll
    for (int i = 0; i < kTileTokens; ++i) {
      const int64_t t = t0 + i;
      const bool live = t >= a.T_old && t < T_new;
      float n = 0.f;
      bool out = false;
      if (live) {
        const float xv = __half2float(xs[i][c]);
        if (KIND == 0) {
          n = normalize(xv, kz, ks);
          out = a.outliers && fabsf(n) >= kt;
        } else {
          n = normalize(xv, s_vz[i], s_vs[i]);
          out = a.outliers && selected(abs_bits(n), (int32_t)cfull, s_rs[i]);
        }
        const float dense = out ? 0.f : fminf(fmaxf(n, -1.f), 1.f);
        const int code = nearest_centroid_sorted(dense, s_cbs, s_cbi, ncb);
        s_code[i][c] = (uint8_t)code;
        // an entry holds the dequantized value at its position (as the emit kernel's)
        if (out)
          n = dequant_ref(s_cb[code], n, KIND == 0 ? ks : s_vs[i], KIND == 0 ? kz : s_vz[i]);
      }
      nval[i] = n;
      if (out) omask |= 1u << i;
      const uint32_t bal = __ballot_sync(0xffffffffu, out);
      if (lane == 0) {
        cnt[i][2 * w] = __popc(bal & 0xffffu);
        cnt[i][2 * w + 1] = __popc(bal >> 16);
      }
    }
    __syncthreads();
    {  // exclusive prefix over (token, 16-channel group): thread c owns entries 2c, 2c+1
      int32_t* flat = &cnt[0][0];
      const int32_t v0 = flat[2 * c], v1 = flat[2 * c + 1];
      int32_t incl = v0 + v1;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t o = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += o;
      }
      if (lane == 31) s_red[w] = incl;
      __syncthreads();
      int32_t base = 0;
      for (int k = 0; k < w; ++k) base += s_red[k];
      const int32_t excl = base + incl - v0 - v1;
      flat[2 * c] = excl;
      flat[2 * c + 1] = excl + v0;
      if (c == 64) s_n0 = excl;  // entries of tokens 0..15 (flat index 128)
      if (c == 127) s_tot = excl + v0 + v1;
    }
    __syncthreads();
    const uint32_t below = (1u << (lane & 15)) - 1u;
#pragma unroll
    for (int i = 0; i < kTileTokens; ++i) {
      const bool out = (omask >> i) & 1u;
      const uint32_t bal = __ballot_sync(0xffffffffu, out);
      if (out) {
        const uint32_t grp = lane < 16 ? (bal & 0xffffu) : (bal >> 16);
        a.out_ent[end + cnt[i][c >> 4] + __popc(grp & below)] = outlier_entry(i, c, nval[i]);
      }
    }
    if (c == 0) {
      const int64_t r0 = urow + 2 * tile;
      if (t0 + 16 > a.T_old) a.out_ptr[r0 + 1] = (int32_t)(end + s_n0);  // block 0 took tokens
      a.out_ptr[r0 + 2] = (int32_t)(end + s_tot);
    }
    // Slabs of the tile, as the emit kernel packs them.
    if (c < 64) {
      const int blk = c >> 5, g = lane >> 2, cc = lane & 3;
      uint32_t slab[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        int ta, ca, tb, cb2;
        slot_map<KIND>(q, blk, g, cc, ta, ca, tb, cb2);
        const uint32_t pair = (uint32_t)s_code[ta][ca] | ((uint32_t)s_code[tb][cb2] << BITS);
        const int bit = 2 * BITS * q;
        slab[bit >> 5] |= pair << (bit & 31);
        if ((bit & 31) + 2 * BITS > 32) slab[(bit >> 5) + 1] |= pair >> (32 - (bit & 31));
      }
      uint8_t* bb = tile_base + blk * (256 * BITS);
      *reinterpret_cast<uint4*>(bb + lane * 16) = make_uint4(slab[0], slab[1], slab[2], slab[3]);
      if (BITS == 4)
        *reinterpret_cast<uint4*>(bb + 512 + lane * 16) = make_uint4(slab[4], slab[5], slab[6], slab[7]);
      else if (BITS == 3)
        *reinterpret_cast<uint2*>(bb + 512 + lane * 8) = make_uint2(slab[4], slab[5]);
    }
    end += s_tot;
    __syncthreads();  // the next tile reuses the shared buffers
  }
}

template <int KIND>
static void launch_append(const AppendArgs& aa, dim3 grid, cudaStream_t st) {
  switch (aa.bits) {
    case 2: append_kernel<KIND, 2><<<grid, 128, 0, st>>>(aa); break;
    case 3: append_kernel<KIND, 3><<<grid, 128, 0, st>>>(aa); break;
    default: append_kernel<KIND, 4><<<grid, 128, 0, st>>>(aa); break;
  }
}

static int check_append(const char* what, const void* x, int64_t B, int64_t S_new,
                        int64_t C_full, int64_t h0, int64_t n_heads, int bits, int64_t T_old,
                        int64_t nt_cap, const void* codes, const int32_t* out_ptr,
                        const uint32_t* out_ent, int64_t ent_stride, const int32_t* status) {
  int rc = check_block(what, B, S_new, C_full, h0, n_heads, nt_cap);
  if (!rc) rc = check_x(what, x, C_full);
  if (rc) return rc;
  if (!bits_ok(bits)) {
    set_error("%s: bits must be 2, 3 or 4 (got %d)", what, bits);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (T_old < 1 || T_old + S_new > (nt_cap - 1) * kTileTokens) {
    set_error("%s: tokens [%lld, %lld) need 1 <= T_old and a spare tile after the last one "
              "(nt_cap=%lld holds %lld appendable positions)", what, (long long)T_old,
              (long long)(T_old + S_new), (long long)nt_cap, (long long)((nt_cap - 1) * kTileTokens));
    return KVQ_ERR_INVALID;
  }
  if (!codes || !out_ptr || !out_ent || !status || ent_stride < 1 ||
      B * n_heads * ent_stride >= (1LL << 31)) {
    set_error("%s: missing cache buffers or invalid ent_stride=%lld", what, (long long)ent_stride);
    return KVQ_ERR_INVALID;
  }
  return KVQ_OK;
}

}  // namespace kvq

extern "C" int kvq_append_keys(const void* k_new, int64_t B, int64_t S_new, int64_t C_full,
                               int64_t h0, int64_t n_heads, const float* scale, const float* zero,
                               const float* thresholds, const float* codebook, int bits,
                               int64_t T_old, uint8_t* codes, int64_t nt_cap, int32_t* out_ptr,
                               uint32_t* out_ent, int64_t ent_stride, int32_t* status,
                               void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_append("append_keys", k_new, B, S_new, C_full, h0, n_heads, bits, T_old, nt_cap,
                        codes, out_ptr, out_ent, ent_stride, status);
  if (rc) return rc;
  if (!scale || !zero || !codebook) {
    set_error("append_keys: scale, zero and codebook are required");
    return KVQ_ERR_INVALID;
  }
  AppendArgs aa{};
  aa.x = (const __half*)k_new; aa.B = B; aa.S_new = S_new; aa.C_full = C_full; aa.h0 = h0;
  aa.H = n_heads; aa.T_old = T_old; aa.k_scale = scale; aa.k_zero = zero; aa.k_thr = thresholds;
  aa.outliers = thresholds != nullptr; aa.cb = codebook; aa.bits = bits; aa.codes = codes;
  aa.nt_cap = nt_cap; aa.out_ptr = out_ptr; aa.out_ent = out_ent; aa.ent_stride = ent_stride;
  aa.status = status;
  launch_append<0>(aa, dim3((unsigned)n_heads, (unsigned)B), as_stream(stream));
  return check_launch("append_keys");
}

extern "C" size_t kvq_append_values_workspace(int64_t B, int64_t S_new) {
  return kvq::value_ws_bytes(B, S_new);
}

extern "C" int kvq_append_values(const void* v_new, int64_t B, int64_t S_new, int64_t C_full,
                                 int64_t h0, int64_t n_heads, double outlier_ratio,
                                 const float* codebook, int bits, int64_t T_old, float* v_scale,
                                 float* v_zero, int64_t ld_stats, uint8_t* codes, int64_t nt_cap,
                                 int32_t* out_ptr, uint32_t* out_ent, int64_t ent_stride,
                                 void* workspace, size_t workspace_bytes, int32_t* status,
                                 void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_append("append_values", v_new, B, S_new, C_full, h0, n_heads, bits, T_old,
                        nt_cap, codes, out_ptr, out_ent, ent_stride, status);
  if (rc) return rc;
  if (C_full > kValRowMax) {
    set_error("append_values: C=%lld channels exceed %d", (long long)C_full, kValRowMax);
    return KVQ_ERR_UNSUPPORTED;
  }
  if (!v_scale || !v_zero || !codebook || ld_stats < T_old + S_new) {
    set_error("append_values: missing stats / codebook or ld_stats=%lld < %lld tokens",
              (long long)ld_stats, (long long)(T_old + S_new));
    return KVQ_ERR_INVALID;
  }
  if (!workspace || workspace_bytes < value_ws_bytes(B, S_new)) {
    set_error("append_values: workspace too small");
    return KVQ_ERR_INVALID;
  }
  cudaStream_t st = as_stream(stream);
  Select* sel = reinterpret_cast<Select*>(workspace);
  const bool outliers = outlier_ratio > 0;
  const int64_t kv = outliers ? outlier_count(C_full, outlier_ratio) : 0;
  // Per-token stats and top-k of the new rows (no sink: every new token is quantized).
  const size_t smem = C_full * sizeof(uint32_t);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(value_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  value_plan_kernel<<<(unsigned)(B * S_new), plan_threads(C_full), smem, st>>>(
      (const __half*)v_new, B, S_new, C_full, 0, kv, v_scale + T_old, v_zero + T_old, ld_stats,
      sel, nullptr, 0, 0, 0);
  AppendArgs aa{};
  aa.x = (const __half*)v_new; aa.B = B; aa.S_new = S_new; aa.C_full = C_full; aa.h0 = h0;
  aa.H = n_heads; aa.T_old = T_old; aa.v_scale = v_scale; aa.v_zero = v_zero;
  aa.ld_stats = ld_stats; aa.sel = sel; aa.outliers = outliers; aa.cb = codebook; aa.bits = bits;
  aa.codes = codes; aa.nt_cap = nt_cap; aa.out_ptr = out_ptr; aa.out_ent = out_ent;
  aa.ent_stride = ent_stride; aa.status = status;
  launch_append<1>(aa, dim3((unsigned)n_heads, (unsigned)B), st);
  return check_launch("append_values");
}
