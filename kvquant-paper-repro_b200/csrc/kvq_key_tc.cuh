// Key kernel on the fifth-generation tensor cores (tcgen05, TMEM accumulators)
// for one query head per KV head. Part of the kvq_lib.cu unity build.
//
// Same arithmetic as key_scores_kernel (kvq_decode.cuh): per RoPE pair p
// (channels p, p+64) with code values L1, L2,
//   X = L1*(s1 q1) + L2*(s2 q2) + (z1 q1 + z2 q2)
//   Y = L1*(s1 q2) - L2*(s2 q1) + (z1 q2 - z2 q1)
//   score += cos(t th_p) * X + sin(t th_p) * Y
// with fp32 angles fl(t * inv_freq) (kvquant/kernels/rope_fused.py:6-12) and the
// dequantization (cb[code] + o) * s + z of kvquant/quant/kv_quantizer.py:89.
//
// Work item = (group of up to 8 units, M-tile of 128 tokens = 4 code tiles).
// Per unit the CTA forms X and Y for all 128 tokens x 64 pairs as one
// tcgen05.mma sequence, M = 128 tokens:
//   * A (TMEM, 128 lanes x 64 columns) = the fp16 code values, written by the
//     eight block warps (one 16-token block each) with tcgen05.st.16x256b from
//     the pair LUT. The cache's lane slabs are already in that store's
//     register order: a lane's slab pair q is token g + 8(q & 1), RoPE pair
//     4(q >> 1) + c (lane = 4g + c), and TMEM column 8*rep + 2c + j of the
//     store is that pair with q = 4*rep + 2j + r.
//   * B (shared memory, per unit) = the block-diagonal per-head constants
//     divided by a power of two sigma: step s covers pairs 8s..8s+7 (K = 16
//     channels, N = 16 outputs X/Y); a zero-point MMA (N = 128, K = 16, a
//     constant A column of 256 times the terms / 256 split into fp16 high and
//     low parts) writes the zero-point terms first.
//   * D (TMEM, 128 lanes x 128 fp32 columns) = X, Y of every (token, pair).
//     A block warp reads its 16 lanes back with tcgen05.ld.16x256b: lane
//     4g + c receives X, Y of pairs 4kb + c for tokens g, g + 8 -- the pairs
//     whose exact-angle cos/sin it holds in registers for the whole item.
// Outliers add (d - dense) (cos qa + sin qb) / sigma per entry (exact trig; d =
// the entry's dequantized key, dense = the MMA's cb[c0] s + z) into per-token
// 64-bit fixed-point shared-memory sums (integer atomics, no float CAS loop).
// Pipeline: a copy warp streams each unit's 128-token code slab with bulk
// copies into a ring that fills the rest of shared memory (up to 24 stages);
// an MMA warp issues the MMAs into one of two TMEM A buffers and three D
// buffers; the block warps dequantize the next unit into A while running the
// rotation epilogue of a unit two behind. Every mbarrier wait is bounded in
// time, sets an abort flag and status bit 2, and the kernel frees its TMEM.
// This kernel keeps single fp16 code values and constants (the mma.sync key
// kernel splits both into high and low parts).
#pragma once
#include <atomic>
#include <cstdlib>

#include "kvq_decode.cuh"
#include "kvq_sm100.cuh"

namespace kvq {

constexpr int kTcBlockWarps = 8;                       // 16-token blocks per M-tile
constexpr int kTcMmaWarp = kTcBlockWarps;              // issues the MMAs, rebuilds tables
constexpr int kTcCopyWarp = kTcBlockWarps + 1;         // streams the code tiles
constexpr int kTcThreads = (kTcBlockWarps + 2) * 32;
constexpr int kTcTiles = 4;                            // 32-token code tiles per M-tile
constexpr int kTcTokens = kTcTiles * kTileTokens;      // 128
constexpr int kTcMaxUnits = 8;                         // units per group
constexpr uint32_t kTcCols = 512;                      // TMEM columns
constexpr uint32_t kTcA = 0;                           // A buffers: [0, 64), [64, 128)
constexpr uint32_t kTcD = 128;                         // D buffers: [128, 256), [256, 384), [384, 512)
constexpr int kTcDBufs = 3;
constexpr uint32_t kTcIdescStep = sm100::idesc_f16_f32(128, 16);
constexpr uint32_t kTcIdescZero = sm100::idesc_f16_f32(128, 128);

template <int BITS>
struct KeyTcSmem {
  static constexpr int kBlockBytes = 256 * BITS;                 // one 16-token block of a unit
  static constexpr int kStageBytes = kTcTiles * 2 * kBlockBytes;  // one unit's M-tile
  static constexpr int kBMain = PairLut<BITS>::kBytes;           // [unit][step][512 B]
  static constexpr int kBZero = kBMain + kTcMaxUnits * 4096;     // [unit][2048 B]
  static constexpr int kZeros = kBZero + kTcMaxUnits * 2048;     // 2048 B of zeros
  static constexpr int kAConst = kZeros + 2048;                  // 128 x 16 fp16: K 0, 1 = 256
  static constexpr int kPQ = kAConst + 4096;                     // [unit][128] float2 (qa, qb) / sigma
  static constexpr int kDense = kPQ + kTcMaxUnits * 1024;        // [unit][128] float cb[c0] s + z
  static constexpr int kSigma = kDense + kTcMaxUnits * 512;      // [unit] float
  static constexpr int kSink = kSigma + kTcMaxUnits * 4;         // [unit] float, sink score / sigma
  static constexpr int kInv = kSink + kTcMaxUnits * 4;           // [64] float
  static constexpr int kSlots = kInv + kPairs * 4;               // [warp][16] u64 outlier sums
  static constexpr int kBars = kSlots + kTcBlockWarps * 16 * 8;
  // codes_full[S], codes_empty[S], a_full[2], d_empty[3], mma_done[3], drained, tables;
  // the code ring fills the rest of shared memory (up to 24 stages)
  static constexpr int kFixed = kBars + (2 * 24 + 10) * 8 + 16;
  static constexpr int kStagesFit = (232448 - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit > 24 ? 24 : kStagesFit;
  static constexpr int kNumBars = 2 * kStages + 10;
  static constexpr int kTmemPtr = kBars + kNumBars * 8;
  static constexpr int kAbort = kTmemPtr + 4;
  static constexpr int kRing = (kAbort + 12 + 127) / 128 * 128;
  static constexpr int kBytes = kRing + kStages * kStageBytes;
  static_assert(kStages >= 4, "key code ring");
  static_assert(kBytes <= 232448, "tcgen05 key kernel shared memory");
  static_assert(kBars % 8 == 0 && kRing % 16 == 0 && kBMain % 16 == 0 && kAConst % 16 == 0,
                "alignment");
};

template <int BITS>
__host__ __device__ constexpr int key_tc_smem_bytes() { return KeyTcSmem<BITS>::kBytes; }

// Position of flat unit j of a CTA's sequence: item (group, M-tile) and unit in group.
struct TcCursor {
  int64_t w;   // work item
  int ui;      // unit within the group
  int nu;      // units in this item's group
};

__device__ __forceinline__ void tc_cursor_begin(TcCursor& cur, int64_t w, int n_mt, int UG,
                                                int64_t U) {
  cur.w = w;
  cur.ui = 0;
  const int64_t grp = w / n_mt;
  cur.nu = (int)min((int64_t)UG, U - grp * UG);
}
__device__ __forceinline__ void tc_cursor_next(TcCursor& cur, int n_mt, int UG, int64_t U) {
  if (++cur.ui >= cur.nu) tc_cursor_begin(cur, cur.w + 1, n_mt, UG, U);
}

// Builds the B tables, (P, Q) table, sigma and sink scores of a group (units
// u0 .. u0 + nu - 1) with the threads [t0, t0 + nt) of the CTA; the callers
// order the writes before their readers.
template <int BITS>
__device__ void key_tc_tables(const KeyArgs& a, uint8_t* smem, int64_t u0, int nu, int t0,
                              int nthr) {
  using L = KeyTcSmem<BITS>;
  const int tid = (int)threadIdx.x - t0;
  float* sigma = reinterpret_cast<float*>(smem + L::kSigma);
  float* sink = reinterpret_cast<float*>(smem + L::kSink);
  // zero the B tables (main + zero-point) of nu units
  {
    uint4* z = reinterpret_cast<uint4*>(smem + L::kBMain);
    for (int i = tid; i < nu * 256; i += nthr) z[i] = make_uint4(0, 0, 0, 0);
    uint4* zz = reinterpret_cast<uint4*>(smem + L::kBZero);
    for (int i = tid; i < nu * 128; i += nthr) zz[i] = make_uint4(0, 0, 0, 0);
  }
  // sigma per unit: power of two >= every |s q| product of the head (one warp per unit)
  const int lane = tid & 31, wid = tid >> 5, nw = nthr >> 5;
  for (int ui = wid; ui < nu; ui += nw) {
    const int64_t u = u0 + ui;
    const int64_t b = u / a.H, h = u % a.H;
    const __half* qv = a.q + (b * a.H + h) * kHeadDim;
    const float* scl = a.k_scale + h * kHeadDim;
    float m = 0.f, dot = 0.f;
    for (int p = lane; p < kPairs; p += 32) {
      const float q1 = __half2float(qv[p]), q2 = __half2float(qv[p + 64]);
      const float s1 = scl[p], s2 = scl[p + 64];
      m = fmaxf(m, fmaxf(fmaxf(fabsf(s1 * q1), fabsf(s2 * q2)), fmaxf(fabsf(s1 * q2), fabsf(s2 * q1))));
    }
    m = warp_max(m);
    const float sg = ldexpf(1.f, pow2_exponent(m));
    if (a.k_sink) {
      const __half* kv = a.k_sink + (b * a.H + h) * kHeadDim;
      for (int d = lane; d < kHeadDim; d += 32) dot = fmaf(__half2float(qv[d]), __half2float(kv[d]), dot);
      dot = warp_sum(dot);
    }
    if (lane == 0) {
      sigma[ui] = sg;
      sink[ui] = dot / sg;
    }
  }
}

template <int BITS>
__device__ void key_tc_fill(const KeyArgs& a, uint8_t* smem, int64_t u0, int nu, int t0, int nthr) {
  using L = KeyTcSmem<BITS>;
  const int tid = (int)threadIdx.x - t0;
  const float* sigma = reinterpret_cast<const float*>(smem + L::kSigma);
  float2* pq = reinterpret_cast<float2*>(smem + L::kPQ);
  float* dn = reinterpret_cast<float*>(smem + L::kDense);
  const float cb0 = dense_zero_value(a.cb, 1 << BITS);
  for (int idx = tid; idx < nu * kPairs; idx += nthr) {
    const int ui = idx / kPairs, p = idx % kPairs;
    const int64_t u = u0 + ui;
    const int64_t b = u / a.H, h = u % a.H;
    const __half* qv = a.q + (b * a.H + h) * kHeadDim;
    const float inv = 1.f / sigma[ui];  // a power of two: exact
    const float q1 = __half2float(qv[p]), q2 = __half2float(qv[p + 64]);
    const float s1 = a.k_scale[h * kHeadDim + p], s2 = a.k_scale[h * kHeadDim + p + 64];
    const float z1 = a.k_zero[h * kHeadDim + p], z2 = a.k_zero[h * kHeadDim + p + 64];
    const uint32_t wp = half2_bits(s1 * q1 * inv, s2 * q2 * inv);   // (P1, P2)
    const uint32_t wq = half2_bits(s1 * q2 * inv, -s2 * q1 * inv);  // (Q1, Q2)
    // main B, step s = p >> 3: rows n = 2i (X), 2i + 1 (Y), K columns 2j, 2j + 1
    const int s = p >> 3, i = p & 7, j = 2 * (i & 3) + (i >> 2);
    uint8_t* bs = smem + L::kBMain + ui * 4096 + s * 512;
    const int k = 2 * j;
    const int nx = 2 * i, ny = 2 * i + 1;
    *reinterpret_cast<uint32_t*>(bs + (nx >> 3) * 256 + (k >> 3) * 128 + (nx & 7) * 16 + (k & 7) * 2) = wp;
    *reinterpret_cast<uint32_t*>(bs + (ny >> 3) * 256 + (k >> 3) * 128 + (ny & 7) * 16 + (k & 7) * 2) = wq;
    // zero-point B: D column c = 16 s + 2 i + xy, K = (hi, lo) of term / 256
    uint8_t* bz = smem + L::kBZero + ui * 2048;
    const float ox = (z1 * q1 + z2 * q2) * inv * (1.f / 256.f);
    const float oy = (z1 * q2 - z2 * q1) * inv * (1.f / 256.f);
#pragma unroll
    for (int xy = 0; xy < 2; ++xy) {
      const float term = xy ? oy : ox;
      const __half hi = __float2half_rn(term);
      const __half lo = __float2half_rn(term - __half2float(hi));
      const int c = 16 * s + 2 * i + xy;
      *reinterpret_cast<uint32_t*>(bz + (c >> 3) * 128 + (c & 7) * 16) =
          (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
    }
    // outlier coefficients of channels p and p + 64 (cos, sin factors of the
    // rotated query) and the code tiles' dense value cb[c0] s + z there
    pq[ui * 128 + p] = make_float2(q1 * inv, q2 * inv);
    pq[ui * 128 + p + 64] = make_float2(q2 * inv, -q1 * inv);
    dn[ui * 128 + p] = fmaf(cb0, s1, z1);
    dn[ui * 128 + p + 64] = fmaf(cb0, s2, z2);
  }
}

template <int BITS>
__global__ void __launch_bounds__(kTcThreads, 1) key_scores_tc_kernel(KeyArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  using L = KeyTcSmem<BITS>;
  using namespace sm100;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* codes_full = bars;
  uint64_t* codes_empty = bars + L::kStages;
  uint64_t* a_full = bars + 2 * L::kStages;
  uint64_t* d_empty = a_full + 2;
  uint64_t* mma_done = d_empty + kTcDBufs;
  uint64_t* drained = mma_done + kTcDBufs;
  uint64_t* tables = drained + 1;
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + L::kTmemPtr);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kAbort);
  float* invf = reinterpret_cast<float*>(smem + L::kInv);

  const int64_t U = a.B * a.H;
  const int nt = (int)((a.T + kTileTokens - 1) / kTileTokens);
  const int n_mt = (nt + kTcTiles - 1) / kTcTiles;
  const int UG = a.units_per_group;
  const int64_t w0 = a.n_items * blockIdx.x / gridDim.x;
  const int64_t w1 = a.n_items * (blockIdx.x + 1) / gridDim.x;
  const int64_t tbytes = (int64_t)tile_bytes(BITS);
  const int64_t nblk16 = (a.T + 15) / 16;

  // ---- set-up: LUT, barriers, TMEM, constant A, first group's tables ----
  PairLut<BITS>::build(smem, a.cb);
  if (threadIdx.x < kPairs) invf[threadIdx.x] = a.inv_freq[threadIdx.x];
  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(codes_full + s, 1);
      mbar_init(codes_empty + s, kTcBlockWarps);
    }
    for (int b = 0; b < 2; ++b) mbar_init(a_full + b, kTcBlockWarps);
    for (int b = 0; b < kTcDBufs; ++b) {
      mbar_init(d_empty + b, kTcBlockWarps);
      mbar_init(mma_done + b, 1);
    }
    mbar_init(drained, kTcBlockWarps);
    mbar_init(tables, 1);
    *abort = 0;
    fence_mbar_init();
  }
  {
    uint2* zr = reinterpret_cast<uint2*>(smem + L::kZeros);
    for (int i = threadIdx.x; i < 2048 / 8; i += blockDim.x) zr[i] = make_uint2(0, 0);
    // constant A of the zero-point MMA: every row (K-major core matrices) has K 0, 1 = 256
    uint32_t* ac = reinterpret_cast<uint32_t*>(smem + L::kAConst);
    for (int i = threadIdx.x; i < 4096 / 4; i += blockDim.x)
      ac[i] = ((i & 3) == 0 && ((i >> 5) & 1) == 0) ? kA256 : 0u;
  }
  if (warp == kTcMmaWarp) tmem_alloc(tmem_ptr, kTcCols);
  int64_t cur_grp = w0 < w1 ? w0 / n_mt : -1;
  int cur_nu = 0;
  if (cur_grp >= 0) {
    cur_nu = (int)min((int64_t)UG, U - cur_grp * UG);
    key_tc_tables<BITS>(a, smem, cur_grp * UG, cur_nu, 0, blockDim.x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_ptr;
  if (cur_grp >= 0) key_tc_fill<BITS>(a, smem, cur_grp * UG, cur_nu, 0, blockDim.x);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const int64_t total = [&] {  // units of this CTA's items
    int64_t n = 0;
    for (int64_t w = w0; w < w1; ++w) n += min((int64_t)UG, U - (w / n_mt) * UG);
    return n;
  }();
  if (warp == kTcCopyWarp) {
    // ================= copy warp: keeps every ring stage in flight =================
    TcCursor cc;
    int64_t jc = 0;
    if (w0 < w1) tc_cursor_begin(cc, w0, n_mt, UG, U);
    for (; jc < total; ++jc) {
      const int st = (int)(jc % L::kStages);
      if (jc >= L::kStages &&
          !mbar_wait(codes_empty + st, (uint32_t)(((jc / L::kStages) + 1) & 1), abort))
        break;
      const int64_t grp = cc.w / n_mt;
      const int tile0 = kTcTiles * (int)(cc.w % n_mt);
      const int64_t u = grp * UG + cc.ui;
      const int ntl = min(kTcTiles, nt - tile0);
      if (lane == 0) {
        const uint32_t bytes = (uint32_t)(ntl * tbytes);
        mbar_arrive_expect_tx(codes_full + st, bytes);
        bulk_g2s(smem + L::kRing + st * L::kStageBytes, a.codes + (u * a.nt_cap + tile0) * tbytes,
                 bytes, codes_full + st);
      }
      __syncwarp();
      tc_cursor_next(cc, n_mt, UG, U);
    }
    // drain: every copy issued has landed (bounded) before the CTA exits
    for (int64_t j = (jc > L::kStages ? jc - L::kStages : 0); j < jc; ++j)
      mbar_wait(codes_full + (int)(j % L::kStages), (uint32_t)((j / L::kStages) & 1), abort, false);
  } else if (warp == kTcMmaWarp) {
    // ================= MMA warp =================
    TcCursor cm;
    int64_t jm = 0;
    if (w0 < w1) tc_cursor_begin(cm, w0, n_mt, UG, U);
    int64_t grp_m = cur_grp;
    int n_change = 0;
    bool ok = true;
    const uint32_t ac = smem_addr(smem + L::kAConst);
    const uint32_t zr = smem_addr(smem + L::kZeros);
    while (ok && jm < total) {
      const int64_t grp = cm.w / n_mt;
      if (grp != grp_m) {
        // the block warps' epilogues of the previous group are done: new tables
        if (!mbar_wait(drained, (uint32_t)(n_change & 1), abort)) { ok = false; break; }
        grp_m = grp;
        const int nu = (int)min((int64_t)UG, U - grp * UG);
        key_tc_tables<BITS>(a, smem, grp * UG, nu, kTcMmaWarp * 32, 32);
        __syncwarp();
        key_tc_fill<BITS>(a, smem, grp * UG, nu, kTcMmaWarp * 32, 32);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(tables);
        ++n_change;
      }
      const int ab = (int)(jm & 1), db = (int)(jm % kTcDBufs);
      if (!mbar_wait(a_full + ab, (uint32_t)((jm >> 1) & 1), abort)) { ok = false; break; }
      if (jm >= kTcDBufs &&
          !mbar_wait(d_empty + db, (uint32_t)(((jm / kTcDBufs) + 1) & 1), abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t bm = smem_addr(smem + L::kBMain + cm.ui * 4096);
        const uint32_t bz = smem_addr(smem + L::kBZero + cm.ui * 2048);
        const uint32_t d = tbase + kTcD + 128u * db;
        const uint32_t av = tbase + kTcA + 64u * ab;
        mma_f16_ss(d, smem_desc(ac, 128, 256), smem_desc(bz, zr - bz, 128), kTcIdescZero, 0u);
#pragma unroll
        for (int s = 0; s < 8; ++s)
          mma_f16_ts(d + 16u * s, av + 8u * s, smem_desc(bm + 512u * s, 128, 256), kTcIdescStep, 1u);
        mma_commit(mma_done + db);
      }
      __syncwarp();
      ++jm;
      tc_cursor_next(cm, n_mt, UG, U);
    }
    // drain: every MMA issued has completed (bounded) before the tensor memory is released
    if (jm > 0)
      mbar_wait(mma_done + (int)((jm - 1) % kTcDBufs), (uint32_t)(((jm - 1) / kTcDBufs) & 1), abort,
                false);
  } else {
    // ================= block warps =================
    const int q4 = warp & 3, half = warp >> 2;  // TMEM quadrant, 16-lane half
    const uint32_t lane_off = (uint32_t)(32 * q4 + 16 * half) << 16;
    const int tile_in_mt = q4, blk = half;
    const uint32_t lane4 = (uint32_t)lane << 2;
    const uint8_t* lut = smem;
    unsigned long long* slots = reinterpret_cast<unsigned long long*>(smem + L::kSlots) + warp * 16;
    const float* sigma = reinterpret_cast<const float*>(smem + L::kSigma);
    const float* sinks = reinterpret_cast<const float*>(smem + L::kSink);
    const float2* pqt = reinterpret_cast<const float2*>(smem + L::kPQ);
    const float* dnt = reinterpret_cast<const float*>(smem + L::kDense);

    uint64_t tw[16][2];
    int64_t tw_item = -1;
    int64_t grp_e = cur_grp;  // group whose tables the epilogue reads
    int n_change = 0;
    bool ok = true;

    // units waiting for their epilogue (two behind the one being stored)
    struct Pending {
      int64_t j, w;
      int ui;
      int32_t e0, e1;
      uint32_t ent;
      bool drain;  // the last unit of its group with a unit of another group after it
    };
    Pending pend[2];
    pend[0].j = pend[1].j = -1;

    auto epilogue = [&](Pending& pd) -> bool {
      const int db = (int)(pd.j % kTcDBufs);
      const int64_t grp = pd.w / n_mt;
      const int tile0 = kTcTiles * (int)(pd.w % n_mt);
      if (grp != grp_e) {  // the copy / MMA warp rebuilt the tables for this group
        if (!mbar_wait(tables, (uint32_t)(n_change & 1), abort)) return false;
        grp_e = grp;
        ++n_change;
      }
      const int tok0 = (int)a.pos0 + (tile0 + tile_in_mt) * kTileTokens + 16 * blk;
      if (pd.w != tw_item) {  // the item's exact-angle twiddles: pairs 4kb + c, tokens g, g + 8
        tw_item = pd.w;
#pragma unroll
        for (int kb = 0; kb < 16; ++kb) {
          const float f = invf[4 * kb + c];
          float s0, c0, s8, c8;
          __sincosf(rope_reduce(tok0 + g, f), &s0, &c0);
          __sincosf(rope_reduce(tok0 + g + 8, f), &s8, &c8);
          tw[kb][0] = f2pack(c0, s0);
          tw[kb][1] = f2pack(c8, s8);
        }
      }
      if (!mbar_wait(mma_done + db, (uint32_t)((pd.j / kTcDBufs) & 1), abort)) return false;
      tc_fence_after();
      const uint32_t dad = tbase + kTcD + 128u * db + lane_off;
      // (9 warps: a sub-partition holds three of them, so 168 registers per thread at most;
      // the two halves of D are read one after the other)
      uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};  // token g (kb even, odd), token g + 8 (even, odd)
      uint32_t d[32];
      tmem_ld_16x256b_x8(dad, d);
      tmem_wait_ld();
#pragma unroll
      for (int kb = 0; kb < 8; ++kb) {
        ffma2(acc[kb & 1], tw[kb][0], f2pack(__uint_as_float(d[4 * kb]), __uint_as_float(d[4 * kb + 1])));
        ffma2(acc[2 + (kb & 1)], tw[kb][1],
              f2pack(__uint_as_float(d[4 * kb + 2]), __uint_as_float(d[4 * kb + 3])));
      }
      tmem_ld_16x256b_x8(dad + 64u, d);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_empty + db);
#pragma unroll
      for (int kb = 8; kb < 16; ++kb) {
        const int k8 = kb - 8;
        ffma2(acc[kb & 1], tw[kb][0], f2pack(__uint_as_float(d[4 * k8]), __uint_as_float(d[4 * k8 + 1])));
        ffma2(acc[2 + (kb & 1)], tw[kb][1],
              f2pack(__uint_as_float(d[4 * k8 + 2]), __uint_as_float(d[4 * k8 + 3])));
      }
      float x0 = f2sum(acc[0]) + f2sum(acc[1]), x1 = f2sum(acc[2]) + f2sum(acc[3]);
      x0 += __shfl_xor_sync(0xffffffffu, x0, 1);
      x1 += __shfl_xor_sync(0xffffffffu, x1, 1);
      x0 += __shfl_xor_sync(0xffffffffu, x0, 2);
      x1 += __shfl_xor_sync(0xffffffffu, x1, 2);
      // outliers of the block: (d - dense) * (cos qa + sin qb) / sigma, summed per
      // token in fixed point
      if (pd.e0 < pd.e1) {
        if (lane < 16) slots[lane] = 0ull;
        __syncwarp();
        for (int32_t eb = pd.e0; eb < pd.e1; eb += 32) {
          const int32_t e = eb + lane;
          if (e < pd.e1) {
            const uint32_t en = eb == pd.e0 ? pd.ent : __ldg(a.out_ent + e);
            const int tok = (int)((en >> 7) & 15);
            const int ch = (int)(en & 127), p = ch & 63;
            float sv, cv;
            __sincosf(rope_reduce(tok0 + tok, invf[p]), &sv, &cv);
            const float2 co = pqt[pd.ui * 128 + ch];
            const float v = (entry_value(en) - dnt[pd.ui * 128 + ch]) * fmaf(cv, co.x, sv * co.y);
            atomicAdd(slots + tok, (unsigned long long)__float2ll_rn(v * 4294967296.f));
          }
        }
        __syncwarp();
        x0 += (float)(long long)slots[g] * (1.f / 4294967296.f);
        x1 += (float)(long long)slots[g + 8] * (1.f / 4294967296.f);
        __syncwarp();
      }
      const int64_t u = grp * UG + pd.ui;
      if (tile0 == 0 && tile_in_mt == 0 && blk == 0 && a.k_sink) {
        if (g == 0) x0 = sinks[pd.ui];  // token 0: the fp16 sink, unrotated
      }
      const float sg = sigma[pd.ui];
      x0 *= sg;
      x1 *= sg;
      const int64_t t_blk = (int64_t)(tile0 + tile_in_mt) * kTileTokens + 16 * blk;
      const int64_t row = u;  // one query head per KV head
      if (c < 2) {
        const int64_t tt = t_blk + g + 8 * c;
        if (tt < a.T) a.scores[row * a.T + tt] = c ? x1 : x0;
      }
      if (a.stats && t_blk < a.T) {
        const int64_t tt = t_blk + g + 8 * (c & 1);
        const bool valid = tt < a.T;
        const float v = ((c & 1) ? x1 : x0) * a.stat_scale;
        float m = valid ? v : -INFINITY;
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        float l = valid ? __expf(v - m) : 0.f;
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        if (lane == 0) a.stats[row * nblk16 + t_blk / 16] = make_float2(m, l);
      }
      if (pd.drain) {
        __syncwarp();
        if (lane == 0) mbar_arrive(drained);
      }
      return true;
    };

    int64_t j = 0;
    for (int64_t w = w0; w < w1 && ok; ++w) {
      const int64_t grp = w / n_mt;
      const int tile0 = kTcTiles * (int)(w % n_mt);
      const int nu = (int)min((int64_t)UG, U - grp * UG);
      const int my_tile = tile0 + tile_in_mt;
      const bool next_item_other_group = w + 1 < w1 && (w + 1) / n_mt != grp;
      for (int ui = 0; ui < nu && ok; ++ui, ++j) {
        const int64_t u = grp * UG + ui;
        // this unit's CSR rows (read now, used by its epilogue two iterations later)
        int32_t e0 = 0, e1 = 0;
        if (my_tile < nt) {
          const int64_t r = 2 * (u * a.nt_cap + my_tile) + blk;
          e0 = __ldg(a.out_ptr + r);
          e1 = __ldg(a.out_ptr + r + 1);
        }
        // the oldest pending unit's first entries (its row pointers arrived earlier)
        if (pend[0].j >= 0) {
          const int32_t e = pend[0].e0 + lane;
          pend[0].ent = e < pend[0].e1 ? __ldg(a.out_ent + e) : 0u;
        }
        // code values of this unit's block -> TMEM A
        const int st = (int)(j % L::kStages);
        if (!mbar_wait(codes_full + st, (uint32_t)((j / L::kStages) & 1), abort)) { ok = false; break; }
        const uint8_t* sb = smem + L::kRing + st * L::kStageBytes + tile_in_mt * (2 * L::kBlockBytes) +
                            blk * L::kBlockBytes;
        LaneSlab<BITS> sl;
        sl.read(sb + lane * 16, sb + 512 + lane * (BITS == 4 ? 16 : 8));
        __syncwarp();
        if (lane == 0) mbar_arrive(codes_empty + st);
        uint32_t v[32];
#pragma unroll
        for (int rep = 0; rep < 8; ++rep) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
#pragma unroll
            for (int jj = 0; jj < 2; ++jj)
              v[4 * rep + 2 * r + jj] =
                  *reinterpret_cast<const uint32_t*>(lut + sl.addr(4 * rep + 2 * jj + r, lane4));
          }
        }
        // A buffer j & 1 was read by the MMAs of unit j - 2
        if (j >= 2 && !mbar_wait(mma_done + (int)((j - 2) % kTcDBufs),
                                 (uint32_t)(((j - 2) / kTcDBufs) & 1), abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st_16x256b_x8(tbase + kTcA + 64u * (uint32_t)(j & 1) + lane_off, v);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full + (int)(j & 1));
        if (pend[0].j >= 0 && !epilogue(pend[0])) { ok = false; break; }
        pend[0] = pend[1];
        pend[1].j = j;
        pend[1].w = w;
        pend[1].ui = ui;
        pend[1].e0 = e0;
        pend[1].e1 = e1;
        pend[1].ent = 0u;
        pend[1].drain = ui == nu - 1 && next_item_other_group;
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (ok && pend[k].j >= 0) {
        const int32_t e = pend[k].e0 + lane;
        pend[k].ent = e < pend[k].e1 ? __ldg(a.out_ent + e) : 0u;
        ok = epilogue(pend[k]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kTcMmaWarp) tmem_dealloc(tbase, kTcCols);
}

// One query head per KV head runs on this kernel unless the environment sets
// KVQ_KEY_KERNEL=mma (the mma.sync kernel, kept for group sizes > 1), read once.
// Kernel choice: 0 = warp-level mma.sync kernel (the default), 1 = tcgen05
// kernel. Starts from KVQ_KEY_KERNEL ("tc" selects tcgen05), changed by
// kvq_set_decode_kernels.
inline std::atomic<int>& g_key_kernel() {
  static std::atomic<int> k{[] {
    const char* e = getenv("KVQ_KEY_KERNEL");
    return (e && e[0] == 't') ? 1 : 0;
  }()};
  return k;
}

inline bool use_key_tc() { return g_key_kernel().load(std::memory_order_relaxed) == 1; }

template <int BITS>
static int launch_key_tc(const KeyArgs& a0, cudaStream_t st) {
  KeyArgs a = a0;
  if ((reinterpret_cast<uintptr_t>(a.codes) & 15u) != 0) {
    set_error("key_scores: the code array must be 16-byte aligned");
    return KVQ_ERR_INVALID;
  }
  const int64_t U = a.B * a.H;
  const int64_t nt = (a.T + kTileTokens - 1) / kTileTokens;
  const int64_t n_mt = (nt + kTcTiles - 1) / kTcTiles;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Units per group: up to 16 share an item's RoPE twiddles; short contexts use
  // smaller groups so that every SM gets at least two items.
  int64_t UG = U < kTcMaxUnits ? U : kTcMaxUnits;
  const int64_t want = 2 * (int64_t)sms;
  if (n_mt * ((U + UG - 1) / UG) < want) {
    const int64_t groups = (want + n_mt - 1) / n_mt;
    const int64_t ug = (U + groups - 1) / groups;
    UG = ug < 1 ? 1 : (ug < UG ? ug : UG);
  }
  a.units_per_group = (int)UG;
  a.n_groups = (int)((U + UG - 1) / UG);
  a.n_items = n_mt * a.n_groups;
  const int smem = key_tc_smem_bytes<BITS>();
  cudaFuncSetAttribute(key_scores_tc_kernel<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       smem);
  int64_t grid = sms;
  if (grid > a.n_items) grid = a.n_items;
  if (grid < 1) grid = 1;
  key_scores_tc_kernel<BITS><<<(unsigned)grid, kTcThreads, smem, st>>>(a);
  return check_launch("key_scores");
}

}  // namespace kvq
