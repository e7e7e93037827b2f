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

__device__ __forceinline__ float key_norm(const KeyShape& ks, int64_t b, int64_t t, int64_t c) {
  const float x = __half2float(ks.k[(b * ks.S + t) * ks.C_full + ks.c0 + c]);
  return normalize(x, ks.zero[ks.c0 + c], ks.scale[ks.c0 + c]);
}

constexpr int kHistCols = 32;  // columns per histogram CTA

// Histogram of the radix digit at `shift` of |n| among entries matching the
// prefix so far. grid = (CL/32 column groups, B, row blocks); block 256.
__global__ void __launch_bounds__(256) key_hist_kernel(KeyShape ks, int shift,
                                                       const Select* __restrict__ sel,
                                                       uint32_t* __restrict__ hist,
                                                       int64_t rows_per_block) {
  __shared__ uint32_t h[kHistCols][256];
  for (int i = threadIdx.x; i < kHistCols * 256; i += blockDim.x) (&h[0][0])[i] = 0;
  __syncthreads();
  const int64_t b = blockIdx.y;
  const int64_t cg = (int64_t)blockIdx.x * kHistCols;
  const int lc = threadIdx.x & 31;  // column inside the group
  const int64_t c = cg + lc;
  const int64_t col = b * ks.CL + c;
  const uint32_t mask_hi = shift >= 24 ? 0u : (0xffffffffu << (shift + 8));
  const uint32_t prefix = sel[col].thr & mask_hi;
  const int64_t n_rest = ks.S - ks.off;
  const int64_t r0 = (int64_t)blockIdx.z * rows_per_block;
  const int64_t r1 = min(n_rest, r0 + rows_per_block);
  for (int64_t r = r0 + (threadIdx.x >> 5); r < r1; r += (blockDim.x >> 5)) {
    const uint32_t ab = abs_bits(key_norm(ks, b, r + ks.off, c));
    if ((ab & mask_hi) == prefix) atomicAdd(&h[lc][(ab >> shift) & 0xffu], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kHistCols * 256; i += blockDim.x) {
    const uint32_t v = (&h[0][0])[i];
    if (v) atomicAdd(&hist[(b * ks.CL + cg + i / 256) * 256 + (i & 255)], v);
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

// Columns where only some of the entries equal to thr are taken: one warp per
// such column walks the tokens in order and records the index of the last tie
// taken. Other columns take every tie (tie_cut = INT_MAX).
__global__ void key_ties_kernel(KeyShape ks, Select* __restrict__ sel, int64_t ncols) {
  const int64_t col = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (col >= ncols) return;
  Select s = sel[col];
  if (s.kleft >= s.ties) {
    if (lane == 0) { s.tie_cut = 0x7fffffff; sel[col] = s; }
    return;
  }
  const int64_t b = col / ks.CL, c = col % ks.CL;
  const int64_t n_rest = ks.S - ks.off;
  int32_t need = s.kleft;
  int32_t cut = -1;
  // 256 tokens per step, 8 consecutive ones per lane (8 loads in flight)
  for (int64_t r0 = 0; r0 < n_rest && need > 0; r0 += 256) {
    uint32_t m8 = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int64_t r = r0 + lane * 8 + q;
      if (r < n_rest && abs_bits(key_norm(ks, b, r + ks.off, c)) == s.thr) m8 |= 1u << q;
    }
    const int cnt = __popc(m8);
    int incl = cnt;  // inclusive prefix of the tie counts in token order
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (total >= need) {
      const int L = __ffs(__ballot_sync(0xffffffffu, incl >= need)) - 1;
      const int before = __shfl_sync(0xffffffffu, incl - cnt, L);
      uint32_t m = __shfl_sync(0xffffffffu, m8, L);
      for (int i = 1; i < need - before; ++i) m &= m - 1;  // the (need - before)-th tie of lane L
      cut = (int32_t)(r0 + L * 8 + (__ffs(m) - 1));
      need = 0;
    } else {
      need -= total;
    }
  }
  if (lane == 0) { s.tie_cut = cut; sel[col] = s; }
}

// ---------------------------------------------------------------------------
// Values: one CTA per (b, token) row: per-token min/max over all C_full
// channels, then radix select of the top-k |n| over those channels.
// ---------------------------------------------------------------------------
constexpr int kValRowMax = 16384;  // channels per value row held in smem

__global__ void __launch_bounds__(256) value_plan_kernel(
    const __half* __restrict__ v, int64_t B, int64_t S, int64_t C_full, int64_t off,
    int64_t kv, float* __restrict__ v_scale, float* __restrict__ v_zero, int64_t ld_stats,
    Select* __restrict__ sel) {
  extern __shared__ uint32_t vsm[];  // C_full |n| bits
  __shared__ uint32_t hist[256];
  __shared__ float red_min[8], red_max[8];
  __shared__ int32_t sh_kleft, sh_digit, sh_ties, sh_cut;
  const int64_t row = blockIdx.x;  // over B * (S - off)
  const int64_t n_rest = S - off;
  const int64_t b = row / n_rest, t = row % n_rest + off;
  const __half* x = v + (b * S + t) * C_full;
  float mn = INFINITY, mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < C_full; c += blockDim.x) {
    const float f = __half2float(x[c]);
    mn = fminf(mn, f);
    mx = fmaxf(mx, f);
  }
  mn = -warp_max(-mn);
  mx = warp_max(mx);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { red_min[w] = mn; red_max[w] = mx; }
  __syncthreads();
  if (threadIdx.x < 32) {
    float a = lane < (int)(blockDim.x >> 5) ? red_min[lane] : INFINITY;
    float m2 = lane < (int)(blockDim.x >> 5) ? red_max[lane] : -INFINITY;
    a = -warp_max(-a);
    m2 = warp_max(m2);
    if (lane == 0) { red_min[0] = a; red_max[0] = m2; }
  }
  __syncthreads();
  // kv_quantizer.py:106-107: scale = (max - min) / 2, zero = (max + min) / 2 (fp32).
  const float scale = __fdiv_rn(__fsub_rn(red_max[0], red_min[0]), 2.0f);
  const float zero = __fdiv_rn(__fadd_rn(red_max[0], red_min[0]), 2.0f);
  if (threadIdx.x == 0) {
    v_scale[b * ld_stats + t] = scale;
    v_zero[b * ld_stats + t] = zero;
  }
  for (int64_t c = threadIdx.x; c < C_full; c += blockDim.x)
    vsm[c] = abs_bits(normalize(__half2float(x[c]), zero, scale));
  if (threadIdx.x == 0) sh_kleft = (int32_t)kv;
  __syncthreads();
  uint32_t prefix = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    const uint32_t mask_hi = shift >= 24 ? 0u : (0xffffffffu << (shift + 8));
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int64_t c = threadIdx.x; c < C_full; c += blockDim.x) {
      const uint32_t ab = vsm[c];
      if ((ab & mask_hi) == prefix) atomicAdd(&hist[(ab >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    // The digit holding the k-th largest entry: walking the bins from 255 down,
    // the first d >= 1 whose suffix count reaches k (d = 0 if none). Warp 0:
    // lane L holds bins 8L..8L+7; a suffix scan over the lanes finds the one
    // lane where the count crosses k, which then walks its own 8 bins.
    if (threadIdx.x < 32) {
      const int L = threadIdx.x;
      const int32_t k0 = sh_kleft;
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
        sh_kleft = k;
        sh_digit = d;
        sh_ties = (int32_t)hist[d];
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sh_digit << shift;
    __syncthreads();
  }
  // Tie cut: the channel index of the kleft-th entry equal to the threshold.
  if (threadIdx.x == 0) sh_cut = 0x7fffffff;
  __syncthreads();
  if (sh_kleft < sh_ties) {
    if (threadIdx.x < 32) {
      int32_t need = sh_kleft;
      for (int64_t c0 = 0; c0 < C_full && need > 0; c0 += 32) {
        const int64_t c = c0 + lane;
        const bool tie = c < C_full && vsm[c] == prefix;
        const uint32_t bal = __ballot_sync(0xffffffffu, tie);
        const int cnt = __popc(bal);
        if (cnt >= need) {
          uint32_t m = bal;
          for (int i = 1; i < need; ++i) m &= m - 1;
          if (lane == 0) sh_cut = (int32_t)(c0 + (__ffs(m) - 1));
          need = 0;
        } else {
          need -= cnt;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    Select s;
    s.thr = prefix;
    s.kleft = sh_kleft;
    s.ties = sh_ties;
    s.tie_cut = sh_cut;
    sel[b * S + t] = s;
  }
}

// ---------------------------------------------------------------------------
// Emit: one CTA (128 threads = 4 chunks x 32 tokens) per (b, tile, head).
// KIND 0 = keys, 1 = values. COUNT_ONLY: write the outlier counts of the
// tile's two 16-token blocks into out_ptr[2*(unit*nt_cap + tile) + blk + 1]
// (prefix-summed afterwards into the CSR row pointer over (unit, tile, blk)).
// ---------------------------------------------------------------------------
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
};

// One packed outlier entry: position (token_in_tile << 7 | channel) in the low
// 16 bits, the fp16 normalized value in the high 16 bits.
__device__ __forceinline__ uint32_t outlier_entry(int token, int channel, float value) {
  const __half h = __float2half_rn(value);
  return (uint32_t)((token << 7) | channel) | ((uint32_t)__half_as_ushort(h) << 16);
}

// One CTA of 128 threads per (tile, b, head); thread c owns channel c of the
// head and walks the tile's 32 tokens, so every shared-memory access of a
// warp is to consecutive channels. The tile's fp16 block (32 x 128) is staged
// once with coalesced 16-byte loads; a key channel's zero / scale / selection
// live in registers, a value token's in shared memory.
template <int KIND, bool COUNT_ONLY>
__global__ void __launch_bounds__(128) emit_kernel(EmitArgs a) {
  __shared__ __align__(16) __half xs[kTileTokens][kHeadDim];  // the tile's inputs
  __shared__ int32_t cnt[kTileTokens][8];  // outliers per (token, 16-channel group)
  __shared__ float s_cb[16], s_cbs[16];  // codebook, and sorted ascending
  __shared__ uint8_t s_cbi[16];          // original index of each sorted entry
  __shared__ uint8_t s_code[kTileTokens][kHeadDim];  // codes of the tile (token, channel)
  __shared__ float s_vs[kTileTokens], s_vz[kTileTokens];  // values: per-token scale / zero
  __shared__ Select s_rs[kTileTokens];                   // values: per-token selection
  const int64_t b = blockIdx.y;
  const int64_t tile = blockIdx.x;
  const int64_t h = blockIdx.z;  // local head
  const int c = threadIdx.x;     // channel within the head
  const int lane = c & 31, w = c >> 5;
  const int64_t unit = b * a.H + h;
  const int ncb = 1 << a.bits;
  const int64_t CL = a.H * kHeadDim;
  const int64_t cfull = (a.h0 + h) * kHeadDim + c;
  const int64_t t0 = tile * kTileTokens;
  if (!COUNT_ONLY && c == 0) {
    for (int k = 0; k < ncb; ++k) s_cb[k] = a.cb[k];
    sort_codebook(s_cb, ncb, s_cbs, s_cbi);
  }
  // stage x[t0 .. t0+31][head channels] (rows beyond S read as 0)
  for (int k = c; k < kTileTokens * (kHeadDim / 8); k += 128) {
    const int i = k >> 4, ch8 = (k & 15) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t0 + i < a.S)
      v = *reinterpret_cast<const uint4*>(a.x + (b * a.S + t0 + i) * a.C_full + (a.h0 + h) * kHeadDim + ch8);
    *reinterpret_cast<uint4*>(&xs[i][ch8]) = v;
  }
  float kz = 0.f, ks = 0.f;
  Select cs{};
  if (KIND == 0) {
    kz = a.k_zero[cfull];
    ks = a.k_scale[cfull];
    cs = a.sel[b * CL + h * kHeadDim + c];
  } else if (c < kTileTokens) {
    const int64_t t = t0 + c;
    const bool live = t < a.S && !(a.off == 1 && t == 0);
    s_vs[c] = live ? a.v_scale[b * a.ld_stats + t] : 0.f;
    s_vz[c] = live ? a.v_zero[b * a.ld_stats + t] : 0.f;
    if (live) s_rs[c] = a.sel[b * a.S + t];
  }
  __syncthreads();

  uint32_t omask = 0;  // outlier flag per token i
  float nval[kTileTokens];
#pragma unroll
  for (int i = 0; i < kTileTokens; ++i) {
    const int64_t t = t0 + i;
    const bool is_sink = a.off == 1 && t == 0;
    const bool live = t < a.S && !is_sink;
    float n = 0.f;
    int code = 0;
    bool out = false;
    if (live) {
      const float xv = __half2float(xs[i][c]);
      if (KIND == 0) {
        n = normalize(xv, kz, ks);
        out = a.nnz_cap >= 0 && selected(abs_bits(n), (int32_t)(t - a.off), cs);
      } else {
        n = normalize(xv, s_vz[i], s_vs[i]);
        out = a.nnz_cap >= 0 && selected(abs_bits(n), (int32_t)cfull, s_rs[i]);
      }
      if (!COUNT_ONLY) {
        const float dense = out ? 0.f : fminf(fmaxf(n, -1.f), 1.f);
        code = nearest_centroid_sorted(dense, s_cbs, s_cbi, ncb);
      }
    }
    nval[i] = n;
    if (out) omask |= 1u << i;
    const uint32_t bal = __ballot_sync(0xffffffffu, out);
    if (lane == 0) {
      cnt[i][2 * w] = __popc(bal & 0xffffu);  // channels 32w .. 32w+15
      cnt[i][2 * w + 1] = __popc(bal >> 16);  // channels 32w+16 .. 32w+31
    }
    if (!COUNT_ONLY) {
      s_code[i][c] = (uint8_t)code;
      if (a.dequant_out && t < a.S) {
        __half* drow = a.dequant_out + (b * a.S + t) * CL + h * kHeadDim;
        drow[c] = is_sink ? xs[i][c]
                          : __float2half_rn(dequant_ref(s_cb[code], out ? n : 0.f,
                                                        KIND == 0 ? ks : s_vs[i],
                                                        KIND == 0 ? kz : s_vz[i]));
      }
    }
  }
  if (!COUNT_ONLY && a.sink_out && a.off == 1 && tile == 0) a.sink_out[b * CL + h * kHeadDim + c] = xs[0][c];
  __syncthreads();
  if (COUNT_ONLY) {
    if (c < 2) {  // block c = tokens 16c .. 16c+15
      int32_t tot = 0;
      for (int r = 16 * 8 * c; r < 16 * 8 * (c + 1); ++r) tot += (&cnt[0][0])[r];
      a.out_ptr[2 * (unit * a.nt_cap + tile) + c + 1] = tot;
    }
    return;
  }
  // Exclusive prefix over (token, group) in order -> entry offsets; thread c
  // owns entries 2c, 2c+1 of the 256 (token, group) counts.
  {
    __shared__ int32_t s_wsum[4];
    int32_t* flat = &cnt[0][0];
    const int32_t v0 = flat[2 * c], v1 = flat[2 * c + 1];
    int32_t incl = v0 + v1;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    if (lane == 31) s_wsum[w] = incl;
    __syncthreads();
    int32_t base_w = 0;
    for (int k = 0; k < w; ++k) base_w += s_wsum[k];
    const int32_t excl = base_w + incl - v0 - v1;
    flat[2 * c] = excl;
    flat[2 * c + 1] = excl + v0;
  }
  __syncthreads();
  const int64_t base = a.out_ptr[2 * (unit * a.nt_cap + tile)];  // first entry of the tile
  // Outlier entries in (token, channel) order: rank within the 16-channel group.
  const uint32_t below = (1u << (lane & 15)) - 1u;
#pragma unroll
  for (int i = 0; i < kTileTokens; ++i) {
    const bool out = (omask >> i) & 1u;
    const uint32_t bal = __ballot_sync(0xffffffffu, out);
    if (out) {
      const uint32_t grp = lane < 16 ? (bal & 0xffffu) : (bal >> 16);
      const int64_t e = base + cnt[i][c >> 4] + __popc(grp & below);
      if (e < a.nnz_cap) a.out_ent[e] = outlier_entry(i, c, nval[i]);
    }
  }
  // Slab store: threads 0..63 each pack the slab of (block, lane) = (tid >> 5,
  // tid & 31) in the fragment-native order of the decode kernels.
  if (c < 64) {
    const int blk = c >> 5;
    const int g = lane >> 2, cc = lane & 3;
    uint32_t slab[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // up to 32 bytes (4-bit)
#pragma unroll
    for (int q = 0; q < 32; ++q) {
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
      const uint32_t pair = (uint32_t)s_code[ta][ca] | ((uint32_t)s_code[tb][cb2] << a.bits);
      const int bit = 2 * a.bits * q;
      slab[bit >> 5] |= pair << (bit & 31);
      if ((bit & 31) + 2 * a.bits > 32) slab[(bit >> 5) + 1] |= pair >> (32 - (bit & 31));
    }
    // The block is stored structure-of-arrays: bytes 0..15 of every lane's
    // slab (512 B), then its remaining 8*bits-16 bytes, so that the decode
    // kernels' per-lane copies are coalesced.
    uint8_t* blk_base = a.codes + (unit * a.nt_cap + tile) * (int64_t)tile_bytes(a.bits) +
                        blk * (256 * a.bits);
    *reinterpret_cast<uint4*>(blk_base + lane * 16) = make_uint4(slab[0], slab[1], slab[2], slab[3]);
    if (a.bits == 4)
      *reinterpret_cast<uint4*>(blk_base + 512 + lane * 16) = make_uint4(slab[4], slab[5], slab[6], slab[7]);
    else if (a.bits == 3)
      *reinterpret_cast<uint2*>(blk_base + 512 + lane * 8) = make_uint2(slab[4], slab[5]);
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
inline size_t key_ws_bytes(int64_t B, int64_t n_heads) {
  const int64_t ncols = B * n_heads * kHeadDim;
  return align256(ncols * sizeof(Select)) + align256(ncols * 256 * sizeof(uint32_t));
}
inline size_t value_ws_bytes(int64_t B, int64_t S) {
  return align256((size_t)B * S * sizeof(Select));
}

inline bool bits_ok(int bits) { return bits >= 2 && bits <= 4; }

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
    key_ties_kernel<<<(unsigned)((ncols + 7) / 8), 256, 0, st>>>(ks, sel, ncols);
  }
  // Outlier counts per (unit, tile, block), then the row pointer.
  const int64_t nrows = 2 * B * n_heads * nt_cap;  // (unit, tile, 16-token block)
  zero_i32_kernel<<<grid_for(nrows + 1, 256), 256, 0, st>>>(out_ptr, nrows + 1);
  EmitArgs ea{};
  ea.x = ks.k; ea.B = B; ea.S = S; ea.C_full = C_full; ea.h0 = h0; ea.H = n_heads;
  ea.off = ks.off; ea.k_scale = scale; ea.k_zero = zero; ea.sel = sel; ea.bits = 2;
  ea.nt_cap = nt_cap; ea.out_ptr = out_ptr; ea.nnz_cap = outliers ? 0 : -1;
  const int64_t nt = (S + kTileTokens - 1) / kTileTokens;
  ea.cb = nullptr;  // COUNT_ONLY never reads the codebook
  emit_kernel<0, true><<<dim3((unsigned)nt, (unsigned)B, (unsigned)n_heads), 128, 0, st>>>(ea);
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
  const int64_t tb = tile_bytes(bits);
  if (nt_cap > nt)
    for (int64_t u = 0; u < B * n_heads; ++u)
      cudaMemsetAsync(codes + (u * nt_cap + nt) * tb, 0, (nt_cap - nt) * tb, st);
  EmitArgs ea{};
  ea.x = (const __half*)k; ea.B = B; ea.S = S; ea.C_full = C_full; ea.h0 = h0;
  ea.H = n_heads; ea.off = (sink && S > 1) ? 1 : 0; ea.k_scale = scale; ea.k_zero = zero;
  ea.sel = reinterpret_cast<const Select*>(workspace); ea.cb = codebook; ea.bits = bits;
  ea.codes = codes; ea.nt_cap = nt_cap; ea.out_ptr = const_cast<int32_t*>(out_ptr);
  ea.out_ent = out_ent;
  ea.nnz_cap = outlier_ratio > 0 ? nnz_cap : -1;
  ea.sink_out = (__half*)sink_out; ea.dequant_out = (__half*)dequant_out;
  emit_kernel<0, false><<<dim3((unsigned)nt, (unsigned)B, (unsigned)n_heads), 128, 0, st>>>(ea);
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
  if (B * n_rest > 0) {
    const size_t smem = C_full * sizeof(uint32_t);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(value_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
    value_plan_kernel<<<(unsigned)(B * n_rest), 256, smem, st>>>(
        (const __half*)v, B, S, C_full, off, kv, v_scale, v_zero, ld_stats, sel);
  }
  if (off) {  // the sink token carries no stats
    for (int64_t b = 0; b < B; ++b) {
      cudaMemsetAsync(v_scale + b * ld_stats, 0, sizeof(float), st);
      cudaMemsetAsync(v_zero + b * ld_stats, 0, sizeof(float), st);
    }
  }
  const int64_t nrows = 2 * B * n_heads * nt_cap;  // (unit, tile, 16-token block)
  zero_i32_kernel<<<grid_for(nrows + 1, 256), 256, 0, st>>>(out_ptr, nrows + 1);
  EmitArgs ea{};
  ea.x = (const __half*)v; ea.B = B; ea.S = S; ea.C_full = C_full; ea.h0 = h0;
  ea.H = n_heads; ea.off = off; ea.v_scale = v_scale; ea.v_zero = v_zero;
  ea.ld_stats = ld_stats; ea.sel = sel; ea.cb = nullptr; ea.bits = 2; ea.nt_cap = nt_cap;
  ea.out_ptr = out_ptr; ea.nnz_cap = outliers ? 0 : -1;
  const int64_t nt = (S + kTileTokens - 1) / kTileTokens;
  emit_kernel<1, true><<<dim3((unsigned)nt, (unsigned)B, (unsigned)n_heads), 128, 0, st>>>(ea);
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
  const int64_t tb = tile_bytes(bits);
  if (nt_cap > nt)
    for (int64_t u = 0; u < B * n_heads; ++u)
      cudaMemsetAsync(codes + (u * nt_cap + nt) * tb, 0, (nt_cap - nt) * tb, st);
  EmitArgs ea{};
  ea.x = (const __half*)v; ea.B = B; ea.S = S; ea.C_full = C_full; ea.h0 = h0;
  ea.H = n_heads; ea.off = (sink && S > 1) ? 1 : 0; ea.v_scale = v_scale; ea.v_zero = v_zero;
  ea.ld_stats = ld_stats; ea.sel = reinterpret_cast<const Select*>(workspace);
  ea.cb = codebook; ea.bits = bits; ea.codes = codes; ea.nt_cap = nt_cap;
  ea.out_ptr = const_cast<int32_t*>(out_ptr); ea.out_ent = out_ent;
  ea.nnz_cap = outlier_ratio > 0 ? nnz_cap : -1;
  ea.sink_out = (__half*)sink_out; ea.dequant_out = (__half*)dequant_out;
  emit_kernel<1, false><<<dim3((unsigned)nt, (unsigned)B, (unsigned)n_heads), 128, 0, st>>>(ea);
  return check_launch("quantize_values_emit");
}
