// Value kernel on the fifth-generation tensor cores (tcgen05, TMEM accumulator).
// Part of the kvq_lib.cu unity build.
//
// Same arithmetic as value_kernel (kvq_decode.cuh): out[b, hq, :] =
// sum_t p_t * (s_t * (cb[code] + o) + z_t) with the per-token scale / zero of
// kvquant/quant/kv_quantizer.py:103-117, the dense part as an MMA, outliers,
// zero-point and sink terms in fp32; same work items (unit, split of its tiles)
// and the same fp32 partials [split][row][128 channels + zero term].
//
// Per 128-token chunk of a unit (4 code tiles) the CTA runs 8 MMAs (one per
// 16-token block, K = 16 tokens) of M = 128 channels x N = 16 query heads:
//   * A (TMEM, lanes = channels) = the fp16 code values of V^T. The value
//     tiles are fragment-native for this shape: lane 4g + c of a block holds
//     channels 16mb + g (+8) x tokens 2c, 2c+1 (+8) for every channel block mb,
//     which is tcgen05.st.16x256b's register order for TMEM lanes 16mb..16mb+15.
//     TMEM lanes of quadrant qd belong to warps qd, qd + 4 only, so warp w
//     writes channel blocks 2qd, 2qd + 1 (qd = w & 3) of the chunk's blocks
//     4h .. 4h + 3 (h = w >> 2).
//   * B (shared memory) = the weights p_t * s_t * 2^e in fp16 (e bounds the
//     largest possible weight to 2^14), rows = heads; warp w forms them for
//     block 4h + qd, one token per lane.
//   * D (TMEM, 128 lanes x 16 fp32 columns) accumulates over the split.
// Outliers add p_t s_t o into per-(head, channel) 64-bit fixed-point sums in
// shared memory (integer atomics); the warp that formed a block's weights
// handles the block's entries and passes the weights by shuffle.
// A copy/MMA warp streams the chunks' code tiles by bulk copy through a
// 3-stage ring and issues the MMAs; A and B are double-buffered by chunk.
// Two CTAs share an SM (256 TMEM columns each).
#pragma once
#include <atomic>
#include <cstdlib>

#include "kvq_decode.cuh"
#include "kvq_sm100.cuh"

namespace kvq {

constexpr int kVtWorkers = 8;
constexpr int kVtMmaWarp = kVtWorkers;
constexpr int kVtCopyWarp = kVtWorkers + 1;
constexpr int kVtThreads = (kVtWorkers + 2) * 32;
constexpr int kVtTiles = 4;                       // code tiles per chunk
constexpr int kVtBufs = 3;                        // A / B buffers (chunks in the MMA pipeline)
constexpr uint32_t kVtCols = 512;                 // TMEM: A [0, 384) (three buffers), D [384, 400)
constexpr uint32_t kVtA = 0, kVtD = 384;
constexpr uint32_t kVtACols = 128;                // per buffer: A_hi [0, 64), A_lo [64, 128)
constexpr int kVtMaxG = 8;
constexpr uint32_t kVtIdesc = sm100::idesc_f16_f32(128, 16);

constexpr int kVtEnt = 256;  // outlier entries of a chunk staged in shared memory

template <int BITS, int G>
struct ValTcSmem {
  static constexpr int kBlockBytes = 256 * BITS;
  static constexpr int kStageBytes = kVtTiles * 2 * kBlockBytes;
  // per-chunk side data staged with the codes: scores / probabilities [G][128],
  // scale [128], zero [128], CSR row pointers [9] (+3 pad), entries [kVtEnt]
  static constexpr int kSdP = 0;
  static constexpr int kSdS = kSdP + G * 128 * 4;
  static constexpr int kSdZ = kSdS + 512;
  static constexpr int kSdR = kSdZ + 512;
  static constexpr int kSdE = kSdR + 48;
  static constexpr int kSideBytes = kSdE + kVtEnt * 4;
  static constexpr int kB = PairLutHiLo<BITS>::kBytes;        // [kVtBufs][8 blocks][512 B]
  static constexpr int kAcc = kB + kVtBufs * 8 * 512;          // [G][128] int64 outlier sums
  static constexpr int kZs = kAcc + G * 128 * 8;               // [8 warps][G] float zero terms
  static constexpr int kMl = kZs + kVtWorkers * G * 4;         // [G] float2 (M, 1/L)
  static constexpr int kBars = (kMl + G * 8 + 7) / 8 * 8;
  // codes_full[S], codes_empty[S], a_full[kVtBufs], mma_done[kVtBufs]; the ring
  // (code tiles + side data per stage) fills the rest of shared memory
  static constexpr int kFixed = kBars + (2 * 24 + 2 * kVtBufs) * 8 + 16;
  static constexpr int kStagesFit = (232448 - kFixed - 128) / (kStageBytes + kSideBytes);
  static constexpr int kStages = kStagesFit > 24 ? 24 : kStagesFit;
  static constexpr int kNumBars = 2 * kStages + 2 * kVtBufs;
  static constexpr int kTmemPtr = kBars + kNumBars * 8;
  static constexpr int kAbort = kTmemPtr + 4;
  static constexpr int kRing = (kAbort + 12 + 127) / 128 * 128;
  static constexpr int kSide = kRing + kStages * kStageBytes;
  static constexpr int kBytes = kSide + kStages * kSideBytes;
  static_assert(kStages >= 4, "value code ring");
  static_assert(kBytes <= 232448, "value kernel shared memory");
  static_assert(kB % 16 == 0 && kRing % 16 == 0 && kSide % 16 == 0 && kSideBytes % 16 == 0,
                "alignment");
};

// The 8 code pairs of TMEM quadrant qd (slab slots 8qd .. 8qd + 7, channel
// blocks 2qd and 2qd + 1) of lane `lane`'s slab in a staged block, as a bit
// stream in (hi:lo): pair i at bits [2*BITS*i, 2*BITS*(i + 1)).
template <int BITS>
__device__ __forceinline__ void vt_quadrant_pairs(const uint8_t* blk, int lane, int qd,
                                                  uint32_t& lo, uint32_t& hi) {
  if (BITS == 4) {  // slab bytes 8qd .. 8qd + 7: region 0 holds bytes 0..15, region 1 the rest
    const uint2 w = *reinterpret_cast<const uint2*>(blk + (qd < 2 ? 0 : 512) + lane * 16 +
                                                    8 * (qd & 1));
    lo = w.x;
    hi = w.y;
  } else if (BITS == 2) {  // slab word qd
    lo = *reinterpret_cast<const uint32_t*>(blk + lane * 16 + 4 * qd);
    hi = 0u;
  } else {  // slab bits 48qd .. 48qd + 47 of the 24-byte slab
    const uint4 a = *reinterpret_cast<const uint4*>(blk + lane * 16);
    const uint2 b = *reinterpret_cast<const uint2*>(blk + 512 + lane * 8);
    const uint32_t wa = qd == 0 ? a.x : (qd == 1 ? a.y : (qd == 2 ? a.w : b.x));
    const uint32_t wb = qd == 0 ? a.y : (qd == 1 ? a.z : (qd == 2 ? b.x : b.y));
    const uint32_t sh = (qd & 1) ? 16u : 0u;
    lo = __funnelshift_r(wa, wb, sh);
    hi = wb >> sh;
  }
}

// Pair-LUT byte address of quadrant pair i (0..7) for this lane (lane_off =
// the lane's byte offset within a 256-byte entry row).
template <int BITS>
__device__ __forceinline__ uint32_t vt_pair_addr(uint32_t lo, uint32_t hi, int i, uint32_t lane_off) {
  if (BITS == 4) return prmt(lane_off, i < 4 ? lo : hi, 0x1100u | ((4u + (i & 3)) << 4));
  if (BITS == 2) return (((lo >> (4 * i)) & 15u) << 8) | lane_off;
  const uint64_t v = ((uint64_t)hi << 32) | lo;
  return ((uint32_t)((v >> (6 * i)) & 63u) << 8) | lane_off;
}

template <int BITS, int G>
__global__ void __launch_bounds__(kVtThreads, 1)
    value_tc_kernel(ValueArgs a, const float* __restrict__ row_max) {
  extern __shared__ __align__(16) uint8_t smem[];
  using L = ValTcSmem<BITS, G>;
  using namespace sm100;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* codes_full = bars;
  uint64_t* codes_empty = bars + L::kStages;
  uint64_t* a_full = bars + 2 * L::kStages;
  uint64_t* mma_done = a_full + kVtBufs;
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + L::kTmemPtr);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kAbort);
  unsigned long long* acc = reinterpret_cast<unsigned long long*>(smem + L::kAcc);
  float* zslot = reinterpret_cast<float*>(smem + L::kZs);
  float2* s_ml = reinterpret_cast<float2*>(smem + L::kMl);

  const int nt = (int)((a.T + kTileTokens - 1) / kTileTokens);
  const int T = (int)a.T;
  const int64_t U = a.B * a.H;
  const int64_t u = blockIdx.x / a.n_splits;
  const int split = (int)(blockIdx.x % a.n_splits);
  const int tpb = (nt + a.n_splits - 1) / a.n_splits;
  const int ta = split * tpb, tb = min(nt, ta + tpb);
  const int n_chunks = tb > ta ? (tb - ta + kVtTiles - 1) / kVtTiles : 0;
  const int64_t b = u / a.H, h = u % a.H;
  const int64_t HG = a.H * G;
  const bool sink = a.v_sink != nullptr;
  const float* vs = a.v_scale + b * a.ld;
  const float* vz = a.v_zero + b * a.ld;
  const float* prow = a.probs + (b * HG + h * G) * a.T;
  const int rm_e = pow2_exponent(row_max[b]);
  const float e_scale = ldexpf(1.f, 14 - rm_e);
  const float inv_e = 1.f / e_scale;
  // fixed-point unit of the outlier sums: p s |o| <= row_max <= 2^rm_e (|o| <= 1 for
  // per-token value stats), so 2^(40 - rm_e) keeps every sum within 2^40
  const float fix = ldexpf(1.f, min(100, max(-100, 40 - rm_e)));
  const int64_t tbytes = (int64_t)tile_bytes(BITS);

  // ---- set-up ----
  PairLutHiLo<BITS>::build(smem, a.cb);
  __shared__ float s_cb0;
  if (threadIdx.x == 0) s_cb0 = dense_zero_value(a.cb, 1 << BITS);
  {
    uint4* z = reinterpret_cast<uint4*>(smem + L::kB);
    for (int i = threadIdx.x; i < (kVtBufs * 8 * 512) / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < G * 128; i += blockDim.x) acc[i] = 0ull;
  }
  if (a.ml && threadIdx.x < G) s_ml[threadIdx.x] = a.ml[b * HG + h * G + threadIdx.x];
  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(codes_full + s, 1 + 32);  // the bulk copy's arrival + one per copying lane
      mbar_init(codes_empty + s, kVtWorkers);
    }
    for (int k = 0; k < kVtBufs; ++k) {
      mbar_init(a_full + k, kVtWorkers);
      mbar_init(mma_done + k, 1);
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == kVtMmaWarp) tmem_alloc(tmem_ptr, kVtCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_ptr;

  if (warp == kVtCopyWarp) {
    // ================= copy warp: code tiles + side data, every stage in flight =================
    int jc = 0;
    // this lane's CSR row pointer (lanes 0..8) of chunks jc .. jc + 3, loaded ahead
    auto rp_of = [&](int ch) -> int32_t {
      if (ch >= n_chunks || lane > 8) return 0;
      const int tile0 = ta + kVtTiles * ch;
      const int ntl = min(kVtTiles, tb - tile0);
      return __ldg(a.out_ptr + 2 * (u * a.nt_cap + tile0) + min(lane, 2 * ntl));
    };
    int32_t rpa = rp_of(0), rpb = rp_of(1), rpc = rp_of(2), rpd = rp_of(3);
    auto copy_next = [&]() -> bool {
      const int st = jc % L::kStages;
      if (jc >= L::kStages &&
          !mbar_wait(codes_empty + st, (uint32_t)(((jc / L::kStages) + 1) & 1), abort))
        return false;
      const int tile0 = ta + kVtTiles * jc;
      const int ntl = min(kVtTiles, tb - tile0);
      if (lane == 0) {
        const uint32_t bytes = (uint32_t)(ntl * tbytes);
        mbar_arrive_expect_tx(codes_full + st, bytes);
        bulk_g2s(smem + L::kRing + st * L::kStageBytes, a.codes + (u * a.nt_cap + tile0) * tbytes,
                 bytes, codes_full + st);
      }
      // side data of the chunk's 128 tokens (zero beyond the split and the cache)
      uint8_t* sd = smem + L::kSide + st * L::kSideBytes;
      const int t0 = tile0 * kTileTokens;
      const int tend = min(T, tb * kTileTokens);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int t = t0 + lane + 32 * k;
        const bool in = t < tend;
        const int tc = in ? t : 0;
#pragma unroll
        for (int hd = 0; hd < G; ++hd)
          cp_async_4(sd + L::kSdP + (hd * 128 + lane + 32 * k) * 4, prow + hd * a.T + tc, in ? 4u : 0u);
        cp_async_4(sd + L::kSdS + (lane + 32 * k) * 4, vs + tc, in ? 4u : 0u);
        cp_async_4(sd + L::kSdZ + (lane + 32 * k) * 4, vz + tc, in ? 4u : 0u);
      }
      // row pointers of the chunk's blocks (rows past the split repeat the last one)
      const int64_t r0 = 2 * (u * a.nt_cap + tile0);
      const int64_t rk = r0 + min(lane, 2 * ntl);
      const int32_t rp_lane = rpa;
      rpa = rpb;
      rpb = rpc;
      rpc = rpd;
      rpd = rp_of(jc + 4);
      if (lane <= 8) cp_async_4(sd + L::kSdR + lane * 4, a.out_ptr + rk, 4u);
      const int32_t e_lo = __shfl_sync(0xffffffffu, rp_lane, 0);
      const int32_t e_hi = __shfl_sync(0xffffffffu, rp_lane, 8);
      const int32_t ne = min(e_hi - e_lo, kVtEnt);
      for (int k = lane; k < ne; k += 32)
        cp_async_4(sd + L::kSdE + k * 4, a.out_ent + e_lo + k, 4u);
      cp_async_arrive(codes_full + st);
      ++jc;
      return true;
    };
    for (; jc < n_chunks;)
      if (!copy_next()) break;
    for (int j = (jc > L::kStages ? jc - L::kStages : 0); j < jc; ++j)
      mbar_wait(codes_full + j % L::kStages, (uint32_t)((j / L::kStages) & 1), abort, false);
  } else if (warp == kVtMmaWarp) {
    // ================= MMA warp =================
    int jm = 0;
    for (; jm < n_chunks; ++jm) {
      const int buf = jm % kVtBufs;
      if (!mbar_wait(a_full + buf, (uint32_t)((jm / kVtBufs) & 1), abort)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t bb = smem_addr(smem + L::kB + buf * 4096);
        const uint32_t ab = tbase + kVtA + kVtACols * buf;
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // code values' high parts, then their low parts
          mma_f16_ts(tbase + kVtD, ab + 8u * k, smem_desc(bb + 512u * k, 128, 256), kVtIdesc,
                     (jm > 0 || k > 0) ? 1u : 0u);
          mma_f16_ts(tbase + kVtD, ab + 64u + 8u * k, smem_desc(bb + 512u * k, 128, 256), kVtIdesc,
                     1u);
        }
        mma_commit(mma_done + buf);
      }
      __syncwarp();
    }
    if (jm > 0)
      mbar_wait(mma_done + (jm - 1) % kVtBufs, (uint32_t)(((jm - 1) / kVtBufs) & 1), abort, false);
  } else {
    // ================= worker warps =================
    const int qd = warp & 3, hw = warp >> 2;
    const int wblk = 4 * hw + qd;  // the block whose weights and outliers this warp handles
    const uint32_t lane8 = (uint32_t)lane << 3;
    const uint8_t* lut = smem;
    float zs[G];
#pragma unroll
    for (int hd = 0; hd < G; ++hd) zs[hd] = 0.f;
    const int wt = 16 * wblk + (lane & 15);  // this lane's token of the chunk (lanes 0..15)
    bool ok = true;
    for (int ch = 0; ch < n_chunks && ok; ++ch) {
      const int buf = ch % kVtBufs;
      const int st = ch % L::kStages;
      if (!mbar_wait(codes_full + st, (uint32_t)((ch / L::kStages) & 1), abort)) { ok = false; break; }
      const uint8_t* sd = smem + L::kSide + st * L::kSideBytes;
      // weights of block wblk: p (from the raw score when the stats are given), p s, p z
      const int tile = ta + kVtTiles * ch + (wblk >> 1);
      const int t = tile * kTileTokens + 16 * (wblk & 1) + (lane & 15);
      const bool live = tile < tb && lane < 16 && t < T && !(sink && t == 0);
      const float s_t = live ? reinterpret_cast<const float*>(sd + L::kSdS)[wt] : 0.f;
      const float z_t = live ? reinterpret_cast<const float*>(sd + L::kSdZ)[wt] : 0.f;
      const int32_t* srp = reinterpret_cast<const int32_t*>(sd + L::kSdR);
      const int32_t ebase = srp[0], e0 = srp[wblk], e1 = srp[wblk + 1];
      float p[G], ps[G];
#pragma unroll
      for (int hd = 0; hd < G; ++hd) {
        const float x = reinterpret_cast<const float*>(sd + L::kSdP)[hd * 128 + wt];
        p[hd] = !live ? 0.f
                      : (a.ml ? __expf(x * a.stat_scale - s_ml[hd].x) * s_ml[hd].y : x);
        ps[hd] = p[hd] * s_t;
        zs[hd] = fmaf(p[hd], z_t, zs[hd]);
      }
      // buffers of chunk ch: free once the MMAs of chunk ch - kVtBufs are done
      if (ch >= kVtBufs &&
          !mbar_wait(mma_done + buf, (uint32_t)(((ch / kVtBufs) + 1) & 1), abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane < 16) {
        // token tau = lane of the block sits at K index 2j + (tau & 1), j = 2((tau >> 1) & 3) + (tau >> 3)
        const int tau = lane;
        const int k = 2 * (2 * ((tau >> 1) & 3) + (tau >> 3)) + (tau & 1);
        __half* bw = reinterpret_cast<__half*>(smem + L::kB + buf * 4096 + wblk * 512);
        // rows 0..G-1: the weights' fp16 high parts; rows 8..8+G-1: their low parts
#pragma unroll
        for (int hd = 0; hd < G; ++hd) {
          const float wv = ps[hd] * e_scale;
          const __half wh = __float2half_rn(wv);
          bw[((k >> 3) * 128 + hd * 16 + (k & 7) * 2) / 2] = wh;
          bw[(256 + (k >> 3) * 128 + hd * 16 + (k & 7) * 2) / 2] =
              __float2half_rn(wv - __half2float(wh));
        }
      }
      fence_proxy_async_smem();
      // codes of blocks 4hw .. 4hw + 3, channel blocks 2qd, 2qd + 1 -> TMEM A
      const uint8_t* sb = smem + L::kRing + st * L::kStageBytes;
      uint32_t qlo[4], qhi[4];  // the quadrant's code pairs of blocks 4hw .. 4hw + 3
#pragma unroll
      for (int rep = 0; rep < 4; ++rep)
        vt_quadrant_pairs<BITS>(sb + (4 * hw + rep) * L::kBlockBytes, lane, qd, qlo[rep], qhi[rep]);
      const uint32_t acol = tbase + kVtA + kVtACols * buf + 32u * hw;
#pragma unroll
      for (int m = 0; m < 2; ++m) {  // channel blocks 2qd + m: TMEM lanes 32qd + 16m
        uint32_t vh[16], vl[16];
#pragma unroll
        for (int rep = 0; rep < 4; ++rep) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const uint2 e = *reinterpret_cast<const uint2*>(
                  lut + vt_pair_addr<BITS>(qlo[rep], qhi[rep], 4 * m + r + 2 * jj, lane8));
              vh[4 * rep + 2 * r + jj] = e.x;
              vl[4 * rep + 2 * r + jj] = e.y;
            }
          }
        }
        const uint32_t lanes = (uint32_t)(32 * qd + 16 * m) << 16;
        tmem_st_16x256b_x4(acol + lanes, vh);
        tmem_st_16x256b_x4(acol + 64u + lanes, vl);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full + buf);
      // outliers of block wblk: p_t (d - dense) into (head, channel), fixed point
      const uint32_t* sent = reinterpret_cast<const uint32_t*>(sd + L::kSdE);
      for (int32_t eb = e0; eb < e1; eb += 32) {
        const int32_t e = eb + lane;
        const int32_t rel = e - ebase;
        const uint32_t en = e < e1 ? (rel < kVtEnt ? sent[rel] : __ldg(a.out_ent + e)) : 0u;
        const int tok = (int)((en >> 7) & 15), chn = (int)(en & 127);
        // the entry's dequantized value minus the code tile's cb[c0] s + z there
        const float s_o = __shfl_sync(0xffffffffu, s_t, tok);
        const float z_o = __shfl_sync(0xffffffffu, z_t, tok);
        const float o = entry_value(en) - fmaf(s_cb0, s_o, z_o);
#pragma unroll
        for (int hd = 0; hd < G; ++hd) {
          const float w = __shfl_sync(0xffffffffu, p[hd], tok);
          if (e < e1)
            atomicAdd(acc + hd * 128 + chn, (unsigned long long)__float2ll_rn(w * o * fix));
        }
      }
      // every lane is done with the stage's side data and codes
      __syncwarp();
      if (lane == 0) mbar_arrive(codes_empty + st);
    }
    // zero terms of the warp's tokens
#pragma unroll
    for (int hd = 0; hd < G; ++hd) {
      const float z = warp_sum(zs[hd]);
      if (lane == 0) zslot[warp * G + hd] = z;
    }
  }
  // ---- epilogue: D + outliers + sink -> partials ----
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp < 4 && n_chunks > 0) {
    if (mbar_wait(mma_done + (n_chunks - 1) % kVtBufs,
                  (uint32_t)(((n_chunks - 1) / kVtBufs) & 1), abort, false)) {
      tc_fence_after();
      uint32_t d[16];
      tmem_ld_32x32b_x16(tbase + kVtD + ((uint32_t)(32 * warp) << 16), d);
      tmem_wait_ld();
      const int dd = 32 * warp + lane;
#pragma unroll
      for (int hd = 0; hd < G; ++hd) {
        float side = (float)(long long)acc[hd * 128 + dd] / fix;
        if (sink && ta == 0) {
          float p0 = prow[hd * a.T];
          if (a.ml) p0 = __expf(p0 * a.stat_scale - s_ml[hd].x) * s_ml[hd].y;
          side = fmaf(p0, __half2float(a.v_sink[(b * a.H + h) * kHeadDim + dd]), side);
        }
        float* dst = a.partial + ((int64_t)split * (U * G) + u * G + hd) * 129;
        dst[dd] = fmaf(__uint_as_float(d[hd]) + __uint_as_float(d[8 + hd]), inv_e, side);
        if (dd == 0) {
          float z = 0.f;
#pragma unroll
          for (int w = 0; w < kVtWorkers; ++w) z += zslot[w * G + hd];
          dst[128] = z;
        }
      }
    }
  } else if (warp < 4) {  // an empty split: zero partials
    const int dd = 32 * warp + lane;
    for (int hd = 0; hd < G; ++hd) {
      float* dst = a.partial + ((int64_t)split * (U * G) + u * G + hd) * 129;
      dst[dd] = 0.f;
      if (dd == 0) dst[128] = 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kVtMmaWarp) tmem_dealloc(tbase, kVtCols);
}

// Every group size runs on this kernel unless the environment sets
// KVQ_VALUE_KERNEL=mma (the mma.sync kernel), read once.
// Kernel choice: 0 = warp-level mma.sync kernel (the default), 1 = tcgen05
// kernel. Starts from KVQ_VALUE_KERNEL ("tc" selects tcgen05), changed by
// kvq_set_decode_kernels.
inline std::atomic<int>& g_value_kernel() {
  static std::atomic<int> k{[] {
    const char* e = getenv("KVQ_VALUE_KERNEL");
    return (e && e[0] == 't') ? 1 : 0;
  }()};
  return k;
}

inline bool use_value_tc() { return g_value_kernel().load(std::memory_order_relaxed) == 1; }

template <int BITS, int G>
static int launch_value_tc(const ValueArgs& a, const float* row_max, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(a.codes) & 15u) != 0) {
    set_error("value_output: the code array must be 16-byte aligned");
    return KVQ_ERR_INVALID;
  }
  const int smem = ValTcSmem<BITS, G>::kBytes;
  cudaFuncSetAttribute(value_tc_kernel<BITS, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int64_t U = a.B * a.H;
  value_tc_kernel<BITS, G><<<(unsigned)(U * a.n_splits), kVtThreads, smem, st>>>(a, row_max);
  return check_launch("value_output");
}

}  // namespace kvq
