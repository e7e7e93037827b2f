/*
 * kvquant_b200 -- C ABI of the B200 (sm_100a) KVQuant decode-time quantized-KV
 * attention path.
 *
 * Conventions
 *   - Every entry point returns KVQ_OK (0) or an error code; kvq_last_error()
 *     returns a message for the calling thread's last failure.
 *   - All pointers are device pointers unless stated otherwise. fp16 buffers
 *     are passed as void* (IEEE binary16). `stream` is a cudaStream_t (NULL =
 *     legacy default stream). Calls are asynchronous and allocate nothing:
 *     scratch comes from the caller through (workspace, workspace_bytes),
 *     sized by the matching *_workspace() query.
 *   - Layout of the quantized cache (per layer; unit u = b*n_heads + h):
 *       codes    uint8 [U, nt_cap, 512*bits]: tiles of 32 tokens; tile =
 *                2 blocks of 16 tokens, block = one 8*bits-byte slab per
 *                lane (lane = 4g + c) stored structure-of-arrays: bytes 0..15
 *                of the 32 slabs (512 B), then their remaining 8*bits-16
 *                bytes. Slot q (0..31) of a lane's slab is a code pair at
 *                bits [2*bits*q, +2*bits), first code in the low bits.
 *                Keys: kb = q>>1, r = q&1: token 16*blk + g + 8r, channels
 *                (p, p+64) with p = 4kb + c.
 *                Values: mb = q>>2, i = q&3: channel 16mb + g + 8(i&1),
 *                tokens (16blk + 2c + 8(i>>1), that + 1).
 *                (The order of the decode kernels' tensor-core fragments.)
 *       outliers CSR over rows (u, tile, 16-token block), row index
 *                2*(u*nt_cap + tile) + block: ptr int32 [2*U*nt_cap+1] and one
 *                uint32 entry per outlier: low 16 bits = (token_in_tile << 7)
 *                | channel_in_head, high 16 bits = the fp16 normalized raw
 *                value; entries of a row are ordered by (token, channel).
 *       sink     fp16 [B, n_heads*128]: token 0 kept unquantized.
 *       keys:    scale/zero fp32 [n_heads*128] (per channel, calibrated).
 *       values:  scale/zero fp32 [B, ld] (per token, over all C channels).
 *   - head_dim is 128; bits is 2, 3 or 4.
 */
#ifndef KVQUANT_B200_H
#define KVQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVQ_OK 0
#define KVQ_ERR_INVALID 1
#define KVQ_ERR_CUDA 2
#define KVQ_ERR_UNSUPPORTED 3

/* Message of the calling thread's last error ("" if none). */
const char* kvq_last_error(void);
/* ABI version (major*100 + minor). */
int kvq_version(void);

/* ---------------------------------------------------------------------------
 * The reference's four ops (kvquant/kernels/csrc/kvquant_ops.cu:265-270).
 * ------------------------------------------------------------------------- */

/* Replaces rope_apply (kvquant/kernels/csrc/kvquant_ops.cu:156-182):
 * rotate-half RoPE of x [B,H,S,D] fp16 with fp32 tables cos/sin [s_total, D/2]
 * at positions s + pos_offset; out fp16 [B,H,S,D]. */
int kvq_rope_apply(const void* x, const float* cos_tab, const float* sin_tab, void* out,
                   int64_t B, int64_t H, int64_t S, int64_t D, int64_t pos_offset,
                   int64_t s_total, void* stream);

/* Replaces lut_matvec (kvquant/kernels/csrc/kvquant_ops.cu:184-216):
 * out[i] = sum_j (lut[qmat[i,j]]*scale[s] + zero[s]) * vec[j], s = j if
 * per_channel else i. qmat uint8 [N,D]; lut fp16 [lut_size <= 256];
 * scale/zero fp16 [D] or [N]; vec fp16 [D]; out fp16 [N]. */
int kvq_lut_matvec(const uint8_t* qmat, const void* lut, int64_t lut_size, const void* scale,
                   const void* zero, const void* vec, void* out, int64_t N, int64_t D,
                   int per_channel, void* stream);

/* Replaces sparse_matvec_csr (kvquant/kernels/csrc/kvquant_ops.cu:218-241):
 * out[r] = sum_{k in [row_ptr[r], row_ptr[r+1])} values[k] * vec[col_idx[k]].
 * row_ptr int32 [R+1]; col_idx int32 [nnz]; values/vec/out fp16. Entries
 * whose column is outside [0, vec_len) are skipped and make the call fail
 * with KVQ_ERR_INVALID at the next kvq_check_status(). */
int kvq_sparse_matvec_csr(const int32_t* row_ptr, const int32_t* col_idx, const void* values,
                          const void* vec, void* out, int64_t R, int64_t nnz, int64_t vec_len,
                          void* stream);

/* The normalization step of quantize_k / quantize_v (kvquant/quant/
 * kv_quantizer.py:82,104): out = (x - zero) / (scale + 1e-8), each step an IEEE
 * fp32 operation, computed as the quantize kernels compute it (from the
 * correctly rounded reciprocal of the divisor with two corrections; results
 * equal the IEEE quotient). x fp16 [rows, cols]; zero / scale fp32 [cols]
 * (per_channel != 0) or [rows]; out fp32 [rows, cols]. */
int kvq_normalize(const void* x, int64_t rows, int64_t cols, const float* zero,
                  const float* scale, int per_channel, float* out, void* stream);

/* Replaces lut_lookup (kvquant/kernels/csrc/kvquant_ops.cu:243-263):
 * nearest centroid (first minimum) of x fp32 [N] in codebook fp32 [lut_size];
 * idx_out int64 [N], dq_out fp32 [N]. */
int kvq_lut_lookup(const float* x, const float* codebook, int64_t lut_size, int64_t* idx_out,
                   float* dq_out, int64_t N, void* stream);

/* ---------------------------------------------------------------------------
 * Quantize-on-append (prefill block). Semantics of KVQuantizer.quantize_k /
 * quantize_v (kvquant/quant/kv_quantizer.py:72-122) with dense-and-sparse
 * outliers (kvquant/quant/dense_sparse.py:4-32): codes and outlier positions
 * match the reference bit for bit (ties at the top-k threshold: lower token /
 * channel index wins); each outlier entry holds the reference's fp16
 * dequantized value at its position, fp16((cb[c0] + n) * s + z).
 *
 * Input x [B, S, C_full] fp16 (the k_proj / v_proj output); the call handles
 * heads [h0, h0+n_heads). Token 0 becomes the fp16 sink when sink && S > 1.
 * Two phases: *_plan computes thresholds, per-(unit,tile) outlier counts,
 * out_ptr and the total nnz (device int64); *_emit writes the codes, outlier
 * entries, sink and (optionally) the fake-quant dequantized output
 * [B, S, n_heads*128] fp16 -- the reference's return value. The workspace
 * carries the plan's selections and outlier bounds to the emit call, which
 * also writes its per-channel / per-token code bounds into it (so it is not
 * read-only to *_emit despite the const).
 * ------------------------------------------------------------------------- */
size_t kvq_quantize_keys_workspace(int64_t B, int64_t S, int64_t n_heads);
int kvq_quantize_keys_plan(const void* k, int64_t B, int64_t S, int64_t C_full, int64_t h0,
                           int64_t n_heads, const float* scale, const float* zero,
                           double outlier_ratio, int sink, int32_t* out_ptr, int64_t nt_cap,
                           int64_t* nnz_out, void* workspace, size_t workspace_bytes,
                           void* stream);
int kvq_quantize_keys_emit(const void* k, int64_t B, int64_t S, int64_t C_full, int64_t h0,
                           int64_t n_heads, const float* scale, const float* zero,
                           const float* codebook, int bits, double outlier_ratio, int sink,
                           uint8_t* codes, int64_t nt_cap, const int32_t* out_ptr,
                           uint32_t* out_ent, int64_t nnz_cap, void* sink_out,
                           void* dequant_out, const void* workspace, size_t workspace_bytes,
                           void* stream);

size_t kvq_quantize_values_workspace(int64_t B, int64_t S, int64_t n_heads);
int kvq_quantize_values_plan(const void* v, int64_t B, int64_t S, int64_t C_full, int64_t h0,
                             int64_t n_heads, double outlier_ratio, int sink, float* v_scale,
                             float* v_zero, int64_t ld_stats, int32_t* out_ptr, int64_t nt_cap,
                             int64_t* nnz_out, void* workspace, size_t workspace_bytes,
                             void* stream);
int kvq_quantize_values_emit(const void* v, int64_t B, int64_t S, int64_t C_full, int64_t h0,
                             int64_t n_heads, const float* codebook, int bits,
                             double outlier_ratio, int sink, const float* v_scale,
                             const float* v_zero, int64_t ld_stats, uint8_t* codes,
                             int64_t nt_cap, const int32_t* out_ptr, uint32_t* out_ent,
                             int64_t nnz_cap, void* sink_out,
                             void* dequant_out, const void* workspace, size_t workspace_bytes,
                             void* stream);

/* ---------------------------------------------------------------------------
 * Decode-time append: quantizes S_new new tokens [B, S_new, C_full] fp16 into
 * an existing cache holding T_old >= 1 tokens, at positions T_old.. . The
 * reference re-runs quantize_k / quantize_v on each new block through its
 * k_proj / v_proj hooks (kvquant/attention_patch.py:22-35); these calls keep
 * that per-step semantics for values and give keys the calibrated-threshold
 * outliers of the KVQuant paper (section 3.4), O(S_new) work per call.
 *
 * Layout requirements (kvquant.kernels.make_appendable builds them): a spare
 * tile after the last token (T_old + S_new <= (nt_cap - 1) * 32), and per-unit
 * outlier segments: unit u owns entries [u*ent_stride, (u+1)*ent_stride) and
 * its row pointers address that range. A unit whose segment cannot take the
 * new outliers is left untouched and bit 0 of *status (a device int32) is set;
 * the caller clears *status and reads it after the call.
 * ------------------------------------------------------------------------- */

/* Keys (kv_quantizer.py:72-94 with per-channel thresholds): n = (k - zero) /
 * (scale + 1e-8); |n| >= thresholds[c] is an outlier (fp16 entry, dense part
 * 0), the rest is clamped to [-1, 1] and coded by the first nearest centroid.
 * scale, zero and thresholds are fp32 [n_heads*128], the cache's own channels
 * (heads h0.. of k_new); thresholds NULL = no outliers. thresholds = 0 makes
 * every channel an outlier: the reference's quantize_k on a one-token block. */
int kvq_append_keys(const void* k_new, int64_t B, int64_t S_new, int64_t C_full, int64_t h0,
                    int64_t n_heads, const float* scale, const float* zero,
                    const float* thresholds, const float* codebook, int bits, int64_t T_old,
                    uint8_t* codes, int64_t nt_cap, int32_t* out_ptr, uint32_t* out_ent,
                    int64_t ent_stride, int32_t* status, void* stream);

/* Values (kv_quantizer.py:96-122, each new token as a one-token call: no
 * sink): writes v_scale / v_zero [B, ld_stats] at positions T_old.., codes and
 * entries. Workspace: kvq_append_values_workspace(B, S_new) bytes. */
size_t kvq_append_values_workspace(int64_t B, int64_t S_new);
int kvq_append_values(const void* v_new, int64_t B, int64_t S_new, int64_t C_full, int64_t h0,
                      int64_t n_heads, double outlier_ratio, const float* codebook, int bits,
                      int64_t T_old, float* v_scale, float* v_zero, int64_t ld_stats,
                      uint8_t* codes, int64_t nt_cap, int32_t* out_ptr, uint32_t* out_ent,
                      int64_t ent_stride, void* workspace, size_t workspace_bytes,
                      int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * Decode attention over the packed cache (T cached tokens at positions
 * 0..T-1, token 0 = sink). q fp16 [B, n_heads*group, 128] (already rotated
 * to its own position); query head hq reads KV head hq / group. codes must be
 * 16-byte aligned (tiles are staged with 16-byte copies); a null or unaligned
 * codes pointer returns KVQ_ERR_INVALID before any launch.
 * ------------------------------------------------------------------------- */

/* Fused key kernel: scores[b,hq,t] = q . RoPE_t(Khat_t) (raw, unscaled) fp32
 * [B, n_heads*group, T]. inv_freq fp32 [64] (rope_fused.py:7-8). */
int kvq_key_scores(const uint8_t* codes, const uint32_t* out_ent,
                   const int32_t* out_ptr, const float* k_scale, const float* k_zero,
                   const void* k_sink, const float* codebook, int bits, const void* q,
                   const float* inv_freq, int64_t B, int64_t n_heads, int64_t group,
                   int64_t T, int64_t nt_cap, float* scores, void* stream);

/* probs = softmax(scores * scale) along the last axis; rows x T fp32. */
size_t kvq_softmax_workspace(int64_t rows, int64_t T);
int kvq_softmax(const float* scores, int64_t rows, int64_t T, float scale, float* probs,
                void* workspace, size_t workspace_bytes, void* stream);

/* Value kernel: out[b,hq,:] = sum_t probs[b,hq,t] * Vhat_t (fp16 [B, Hq, 128]). */
size_t kvq_value_output_workspace(int64_t B, int64_t n_heads, int64_t group, int64_t T);
int kvq_value_output(const uint8_t* codes, const uint32_t* out_ent,
                     const int32_t* out_ptr, const float* v_scale, const float* v_zero,
                     int64_t ld_stats, const void* v_sink, const float* codebook, int bits,
                     const float* probs, int64_t B, int64_t n_heads, int64_t group, int64_t T,
                     int64_t nt_cap, void* out, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Softmax fused into the key and value kernels (no counterpart in the
 * reference, which materializes the probabilities; the result is the same
 * softmax). kvq_key_scores_stats is kvq_key_scores that also writes, for
 * every row and 16-token block k of the token axis, stats[row, k] = (m, l):
 * m = max of scores*scale over the block, l = sum of exp(scores*scale - m);
 * stats is fp32 pairs [B*n_heads*group, ceil(T/16)] (kvq_key_stats_size
 * bytes). kvq_value_output_scores takes the raw scores and those stats in
 * place of probabilities and forms softmax(scores * scale) itself (its
 * workspace: kvq_value_output_scores_workspace bytes); it reads `scores` and
 * `stats` and writes neither. */
size_t kvq_key_stats_size(int64_t rows, int64_t T);
size_t kvq_value_output_scores_workspace(int64_t B, int64_t n_heads, int64_t group, int64_t T);
int kvq_key_scores_stats(const uint8_t* codes, const uint32_t* out_ent,
                         const int32_t* out_ptr, const float* k_scale, const float* k_zero,
                         const void* k_sink, const float* codebook, int bits, const void* q,
                         const float* inv_freq, int64_t B, int64_t n_heads, int64_t group,
                         int64_t T, int64_t nt_cap, float* scores, float scale, void* stats,
                         void* stream);
int kvq_value_output_scores(const uint8_t* codes, const uint32_t* out_ent,
                            const int32_t* out_ptr, const float* v_scale, const float* v_zero,
                            int64_t ld_stats, const void* v_sink, const float* codebook,
                            int bits, const float* scores, const void* stats, float scale,
                            int64_t B, int64_t n_heads, int64_t group, int64_t T,
                            int64_t nt_cap, void* out, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Token-range shards of one decode step (restated; the reference has no decode
 * attention). A cache holding the tokens at positions [pos0, pos0 + T) -- its own
 * token 0 is the sink only when pos0 == 0 -- gives, with the two calls below, its
 * shard's output and the softmax row stats (M, 1/L) of softmax(scores * scale)
 * over its tokens, fp32 pairs [B*n_heads*group]; kvq_merge_shards combines the
 * shards of all ranks into the output over the whole context.
 * kvq_key_scores_stats_at = kvq_key_scores_stats with RoPE positions pos0 + t. */
int kvq_key_scores_stats_at(const uint8_t* codes, const uint32_t* out_ent,
                            const int32_t* out_ptr, const float* k_scale, const float* k_zero,
                            const void* k_sink, const float* codebook, int bits, const void* q,
                            const float* inv_freq, int64_t B, int64_t n_heads, int64_t group,
                            int64_t T, int64_t nt_cap, int64_t pos0, float* scores, float scale,
                            void* stats, void* stream);
/* kvq_value_output_scores that also writes the row stats (M, 1/L) to ml_out. */
int kvq_value_output_scores_ml(const uint8_t* codes, const uint32_t* out_ent,
                               const int32_t* out_ptr, const float* v_scale, const float* v_zero,
                               int64_t ld_stats, const void* v_sink, const float* codebook,
                               int bits, const float* scores, const void* stats, float scale,
                               int64_t B, int64_t n_heads, int64_t group, int64_t T,
                               int64_t nt_cap, void* out, float* ml_out, void* workspace,
                               size_t workspace_bytes, void* stream);
/* out[row] = sum_i w_i o_i[row] / sum_i w_i, w_i = L_i exp(M_i - max_j M_j):
 * o_shards fp16 [n_shards, rows, 128], ml_shards fp32 pairs [n_shards, rows],
 * out fp16 [rows, 128]. */
int kvq_merge_shards(const void* o_shards, const float* ml_shards, int64_t n_shards,
                     int64_t rows, void* out, void* stream);

/* scores -> softmax(scores / sqrt(128)) -> p.V in one call; scores_out and
 * probs_out may be NULL (then they live in the workspace). With probs_out
 * NULL the softmax is fused (kvq_key_scores_stats + kvq_value_output_scores,
 * two launches fewer); with probs_out set the probabilities are written by
 * kvq_softmax. */
size_t kvq_decode_attention_workspace(int64_t B, int64_t n_heads, int64_t group, int64_t T);
int kvq_decode_attention(const uint8_t* k_codes, const uint32_t* k_out_ent,
                         const int32_t* k_out_ptr,
                         const float* k_scale, const float* k_zero, const void* k_sink,
                         const float* k_codebook, const uint8_t* v_codes,
                         const uint32_t* v_out_ent,
                         const int32_t* v_out_ptr, const float* v_scale, const float* v_zero,
                         int64_t ld_stats, const void* v_sink, const float* v_codebook,
                         int bits, const void* q, const float* inv_freq, int64_t B,
                         int64_t n_heads, int64_t group, int64_t T, int64_t nt_cap, void* out,
                         float* scores_out, float* probs_out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* No counterpart in the reference. kvq_value_output without a workspace: the
 * scratch comes from a fixed 4 MiB array owned by the library (one per
 * device), for callers that cannot hand the library device memory of their
 * own -- e.g. a host runtime binding this ABI through a plain FFI with no
 * device allocator, or a decode loop that must not call cudaMalloc (it
 * synchronizes the device) between steps. Same arguments and result as
 * kvq_value_output minus (workspace, workspace_bytes).
 *   - Limit: kvq_value_output_workspace(B, n_heads, group, T) must be at most
 *     4 MiB (4194304 bytes); larger shapes return KVQ_ERR_INVALID with a
 *     message and launch nothing.
 *   - Nothing in the scratch needs to start at zero: the call writes every
 *     byte of it that it reads.
 *   - The first call on each device looks the array's address up
 *     (cudaGetSymbolAddress with that device current) and caches it; make
 *     that first call before any stream capture begins.
 *   - All calls on one device share the array: calls whose work overlaps in
 *     time (other streams, or unordered host threads) race on it; calls in
 *     order on one stream are safe.
 *   - The address cached by the first call belongs to the device's primary
 *     context: it does not survive cudaDeviceReset, and callers that drive
 *     the device through a context other than the primary one must not use
 *     this entry point. */
int kvq_value_output_noalloc(const uint8_t* codes, const uint32_t* out_ent,
                             const int32_t* out_ptr, const float* v_scale, const float* v_zero,
                             int64_t ld_stats, const void* v_sink, const float* codebook,
                             int bits, const float* probs, int64_t B, int64_t n_heads,
                             int64_t group, int64_t T, int64_t nt_cap, void* out, void* stream);

/* ---------------------------------------------------------------------------
 * NUQ codebook fitting (offline calibration).
 * ------------------------------------------------------------------------- */

/* Replaces the KMeans fit of train_nuq_codebook (kvquant/quant/nuq.py:39-44):
 * the 2^bits centres minimising sum_i w_i (x_i - c(x_i))^2 over x [n] fp32
 * with weights w [n] fp32 (>= 0, not all 0). Exact 1-D method: weighted
 * histogram of 8192 bins over [min x, max x], the optimal split of the bins
 * into 2^bits intervals (dynamic programming), then refine_iters (0..64)
 * Lloyd steps on the samples. centres: fp32 [2^bits], ascending.
 * status: int32 [2] (device), written by the call: status[1] = occupied bins;
 * status[0] = 0, or flags with `centres` left unwritten: 2 = a sample is NaN
 * or infinite, 4 = a weight is negative or not finite, 1 (alone) = fewer than
 * 2^bits bins are occupied (the caller applies the reference's few-distinct-
 * values rule, nuq.py:26-37). bits 1..4; n >= 1; workspace 256-byte aligned,
 * kvq_fit_codebook_workspace(n) bytes. The reference's degenerate cases
 * (n = 0, n < 2^bits) are the caller's. */
size_t kvq_fit_codebook_workspace(int64_t n);
int kvq_fit_codebook(const float* x, const float* weights, int64_t n, int bits,
                     int refine_iters, float* centres, void* workspace,
                     size_t workspace_bytes, int32_t* status, void* stream);

/* Decode kernel choice, process-wide (no counterpart in the reference, whose
 * decode is unfused torch ops): 0 = warp-level mma.sync kernels (default),
 * 1 = tcgen05 kernels with TMEM accumulators (key kernel: one query head per
 * KV head; other groups keep the mma.sync key kernel), -1 = leave unchanged.
 * The initial choice comes from the environment variables KVQ_KEY_KERNEL /
 * KVQ_VALUE_KERNEL ("tc" = tcgen05). Both kernels compute the same values to
 * fp32 summation order. kvq_decode_kernels returns key | value << 1. */
int kvq_set_decode_kernels(int key_kernel, int value_kernel);
int kvq_decode_kernels(void);

/* Reads and clears the device-side error flag set by kernels that skip
 * out-of-range accesses (synchronizes `stream`). */
int kvq_check_status(void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KVQUANT_B200_H */
