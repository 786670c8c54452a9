/*
 * C ABI of librecap_b200.so: the corrected sparse attention operator of RECAP on
 * NVIDIA B200 (sm_100a).
 *
 * Conventions
 *  - All pointers are device pointers unless stated otherwise; sizes are element counts.
 *  - bf16 tensors are passed as `void*`, fp16 ones as `void*`, fp32 as `float*`.
 *  - A "bank" is one (batch, head) pair: banks = batch * heads, bank = b * heads + h.
 *  - Geometry derived from (S, n_video) with 128-token blocks:
 *        NB = ceil(S/128), S_pad = 128*NB, nB = ceil(n_video/128),
 *        nB_pad = 128*ceil(nB/128), rows = 128*floor(n_video/128),
 *        dense_start = nB-1 if (n_video % 128 and S > n_video) else nB.
 *  - "Reordered" means the token order [Hilbert-ordered video | text] of
 *    recap/sparse/layout.py; "native" is the model's own order.
 *  - Every entry point returns 0 on success or a RECAP_ERR_* code.  Nothing
 *    synchronises the stream or allocates device memory (except recap_peer_alloc,
 *    the allocator of buffers shared between ranks); scratch buffers come
 *    from the caller.  Kernels that wait on on-chip barriers give up after a
 *    bounded time and record RECAP_STATUS_* in the caller's `status` word
 *    (device int, zero-initialised), which the caller reads after the stream.
 *  - The stream is a cudaStream_t passed as `void*` (NULL = legacy default stream).
 */
#ifndef RECAP_B200_H_
#define RECAP_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RECAP_B200_ABI_VERSION 8

#define RECAP_OK 0
#define RECAP_ERR_SHAPE 1
#define RECAP_ERR_LAUNCH 2
#define RECAP_ERR_DEVICE 3
#define RECAP_ERR_UNSUPPORTED 4
#define RECAP_ERR_SCRATCH_LIMIT 5 /* beyond the fixed scratch of recap_refresh_detail_noalloc */

/* values of the device status word */
#define RECAP_STATUS_TIMEOUT_TMA 101
#define RECAP_STATUS_TIMEOUT_MMA 102
#define RECAP_STATUS_TIMEOUT_SOFTMAX 103
#define RECAP_STATUS_TIMEOUT_PRODUCER 104
#define RECAP_STATUS_TIMEOUT_SELFTEST 106 /* recap_wait_selftest only */

int recap_abi_version(void);

/* Layout gather fused with block pooling.
 * Replaces Layout.reorder (recap/sparse/layout.py:86-90) of Q, K and V and the
 * pool_blocks calls (recap/sparse/pooling.py:10-34) of recap/sparse/attention.py:81-82,173-174.
 *   q, k, v        native [batch, heads, S, D] bf16; element strides (b, h, s) of q, k, v in
 *                  `strides[0..8]` (host array), D contiguous; q or v may be NULL
 *   src_row        [S] int32, native token of reordered row r (Layout._gather_indices fwd)
 *   q_reordered, k_reordered  [banks, S_pad, D] bf16 out (nullable)
 *   v_transposed   [banks, D, S_pad] bf16 out, reordered V transposed (nullable)
 *   q_mean, k_mean, v_mean    [banks, nB, D] fp32 block means over video tokens (nullable)
 *   k_mean_bf16    [banks, nB_pad, D] bf16 (nullable), v_mean_t_bf16 [banks, D, nB_pad] bf16
 *                  (nullable); their padding rows/columns must be zero.
 *   k_centred_t    [banks, D, S_pad] bf16 out (nullable): block-centred video keys k - kbar,
 *                  transposed, zero outside the video tokens (operand of recap_value_key_covariance)
 *   basis, rank, variance, variance_bf16 (nullable together): with a basis U [banks, D, D] fp32
 *                  and 0 < rank < D, rank <= recap_gather_max_rank(), the per-block key
 *                  variances in U folded to `rank` (rotated_leaf_moments_triton + fold_rank,
 *                  recap/kernels/closure_stats.py:192-242, recap/sparse/closure.py:96-104):
 *                  variance [banks, nB, D] fp32, variance_bf16 [banks, nB_pad, D].
 *   k_norm_max     [banks, NB] fp32 out (nullable): the largest |k| over the tokens of each
 *                  128-token block (NB = ceil(S/128)); with it the attention kernels bound
 *                  every logit q.k by |q| * k_norm_max and skip their running-max work.
 *   k_mean_norm    [banks, nB] fp32 out (nullable): |bf16(kbar)| of each video block, the
 *                  same bound for the coarse tail. */
int recap_layout_gather(const void* q, const void* k, const void* v, const int64_t* strides, int batch,
                        int heads, int S, int D, int n_video, const int32_t* src_row, void* q_reordered,
                        void* k_reordered, void* v_transposed, float* q_mean, float* k_mean,
                        float* v_mean, void* k_mean_bf16, void* v_mean_t_bf16, void* k_centred_t,
                        const float* basis, int rank, float* variance, void* variance_bf16,
                        float* k_norm_max, float* k_mean_norm, void* stream);

/* recap_layout_gather for a sequence-parallel layer whose projections stay sharded by token:
 * rank q of n_ranks holds native tokens [q tokens_per_rank, (q + 1) tokens_per_rank), and
 * q_ranks[q] / k_ranks[q] / v_ranks[q] (host arrays of device pointers, one per rank, each
 * 16-byte aligned; other ranks' buffers opened with recap_peer_import) point at head 0 of its
 * first token, with the element strides of `strides` (batch 1).  The pass reads every rank's
 * rows directly, over NVLink for the other GPUs, so the sequence-to-head all-to-all of a
 * Ulysses layer (the exchange around Operator.attend in recap's multi-GPU runs) is this
 * gather's load.  n_ranks in [2, 8] with n_ranks * tokens_per_rank = S.  The caller orders
 * the ranks' writes of their shards before this launch (a collective on the stream). */
int recap_layout_gather_ranks(const void* const* q_ranks, const void* const* k_ranks, const void* const* v_ranks,
                              int n_ranks, int tokens_per_rank, const int64_t* strides, int heads, int S, int D,
                              int n_video, const int32_t* src_row, void* q_reordered, void* k_reordered,
                              void* v_transposed, float* q_mean, float* k_mean, float* v_mean, void* k_mean_bf16,
                              void* v_mean_t_bf16, void* k_centred_t, const float* basis, int rank, float* variance,
                              void* variance_bf16, float* k_norm_max, float* k_mean_norm, void* stream);

/* Largest closure rank the layout pass folds itself (larger ranks: recap_closure_stats). */
int recap_gather_max_rank(void);

/* Floats of scratch `workspace` that recap_value_key_covariance needs. */
int64_t recap_cvk_workspace_floats(int banks, int D, int n_video);

/* Pooled value-key covariance C_vk = sum_t v_t (k_t - kbar_blk(t))^T / n_video on tensor cores,
 * from the layout pass's v_transposed and k_centred_t.
 * Replaces pooled_cross_centered_triton_fp32 (recap/kernels/closure_stats.py:245-290).
 *   cvk [banks, D, D] fp32 out; cvk_bf16 [banks, D, D] bf16 out (nullable). */
int recap_value_key_covariance(const void* v_transposed, const void* k_centred_t, int banks, int S, int D,
                               int n_video, float* workspace, float* cvk, void* cvk_bf16, int* status,
                               void* stream);

/* Top-k block selection.
 * Replaces SparseAttention.head_partition (recap/sparse/attention.py:74-94) with
 * block_proxy_mask (recap/sparse/router.py:10-23): score = (qbar . kbar) * scale in fp32,
 * the `keep` highest-scoring key blocks per query block (ties: lower block index first),
 * then the trailing partial video block selected as a row and a column.
 * nB must not exceed 2048 (the attention kernels' limit); larger calls return RECAP_ERR_SHAPE.
 *   partition      [banks, nB, nB] uint8 (bool) out */
int recap_pool_select(const float* q_mean, const float* k_mean, int banks, int nB, int D, int keep,
                      float scale, int n_video, int block_size, uint8_t* partition, void* stream);

/* out2[0] = sum(new & old), out2[1] = sum(new) over n bytes; int64 device array.
 * Replaces the overlap of the re-selection test, recap/operator.py:288-291 and 425-428. */
int recap_partition_overlap(const uint8_t* new_partition, const uint8_t* old_partition, int64_t n,
                            long long* out2, void* stream);

/* Kernel block mask [banks, NB, NB] uint8 from a partition.
 * Replaces build_kernel_block_mask (recap/kernels/block_sparse.py:52-75). */
int recap_kernel_block_mask(const uint8_t* partition, int banks, int S, int n_video, uint8_t* mask,
                            void* stream);

/* Floats of scratch `workspace` that recap_closure_stats needs. */
int64_t recap_closure_workspace_floats(int banks, int D, int n_video);

/* Moment statistics of the coarse tail, in fp32.
 * Replaces pooled_within_block_scatter (recap/sparse/closure.py:42-73),
 * rotated_leaf_moments_triton (recap/kernels/closure_stats.py:192-242),
 * pooled_cross_centered_triton_fp32 (recap/kernels/closure_stats.py:245-290) and
 * fold_rank (recap/sparse/closure.py:96-104).
 *   scatter        [banks, D, D] out (nullable: not computed)
 *   cvk            [banks, D, D] out, C_vk (nullable); cvk_bf16 its bf16 copy (nullable)
 *   basis          [banks, D, D] fp32 (nullable: no variance)
 *   variance       [banks, nB, D] out, per-block variance in the basis, folded to `rank`
 *                  (rank 0: not folded); variance_bf16 [banks, nB_pad, D] copy (nullable). */
int recap_closure_stats(const void* k_reordered, const void* v_transposed, const float* k_mean, int banks,
                        int S, int D, int n_video, int rank, const float* basis, float* scatter, float* cvk,
                        void* cvk_bf16, float* variance, void* variance_bf16, float* workspace,
                        void* stream);

/* basis_t_bf16[b][n][k] = bf16(basis[b][k][n]): the basis cast of
 * rotated_query_square (recap/sparse/closure.py:84-86) as a K-major MMA operand. */
int recap_basis_prep(const float* basis, int banks, int D, void* basis_t_bf16, void* stream);

/* Corrected coarse tail for the cached rows (< rows), with qsq and drift fused.
 * Replaces SparseAttention.coarse_tail_apply (recap/sparse/attention.py:204-231),
 * build_coarse_tail_plan (recap/sparse/planner.py:12-38), coarse_tail_attention
 * (recap/kernels/coarse_tail.py:194-312), rotated_query_square and value_drift
 * (recap/sparse/closure.py:84-93) and, when old_lse is given, _drift_center
 * (recap/operator.py:148-150).
 *   counts_log     [nB] fp32, ln(tokens of each video block)
 *   out            [banks, rows, D] bf16: coarse output + gate * drift
 *   lse            [banks, rows] fp32
 *   old_lse        [banks, rows] fp32 coarse LSE of the last refresh (nullable); with it,
 *                  center [banks] = mean(lse - old_lse) using center_partial [banks, rows/128].
 *   rank           the closure rank variance_bf16 is folded at (its columns >= rank hold
 *                  one value, recap/sparse/closure.py:96-104); 0: not folded.  A folded
 *                  variance lets the quadratic term run over rank + 2 columns.
 *   k_mean_norm    [banks, nB] from recap_layout_gather (nullable): tiles of block means whose
 *                  logit bound stays within 2^64 of a row's running maximum skip the
 *                  per-tile maximum (the same result up to fp32 rounding).
 * nB_pad must not exceed 2048. */
int recap_coarse_tail(const void* q_reordered, const void* basis_t_bf16, const void* cvk_bf16,
                      const void* k_mean_bf16, const void* variance_bf16, const void* v_mean_t_bf16,
                      const uint8_t* partition, const float* counts_log, const float* k_mean_norm,
                      const float* old_lse, int banks,
                      int S, int D, int n_video, float scale, float theta, int rank, void* out, float* lse,
                      float* center_partial, float* center, int* status, void* stream);

/* Exact attention over the kept 128x128 tiles, with the natural-log LSE per row.
 * Replaces block_sparse_exact (recap/kernels/block_sparse.py:78-139) and, with
 * all_blocks = 1, the dense aten._scaled_dot_product_flash_attention of recap/operator.py:254-256.
 *   out            [banks, S, D] bf16; reordered row r is written at row out_pos[r]
 *                  (out_pos NULL: row r); lse [banks, S] fp32 likewise (nullable).
 *   k_norm_max     [banks, NB] from recap_layout_gather (nullable): with it, key blocks whose
 *                  logit bound |q| * k_norm_max stays within 2^64 of a row's running maximum
 *                  skip the per-block maximum and rescale (the same result up to fp32
 *                  rounding); without it every block takes the exact path. */
int recap_block_sparse_fmha(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                            const uint8_t* partition, const float* k_norm_max, int banks, int S, int D,
                            int n_video, int all_blocks, float scale, const int32_t* out_pos, void* out,
                            float* lse, int* status, void* stream);

/* The two attentions of a REFRESH in one pass: dense attention over every key block and,
 * on the way, the block-sparse head over the partition's kept blocks.  Replaces the dense
 * aten._scaled_dot_product_flash_attention of recap/operator.py:254-256 together with the
 * block_sparse_exact head of recap/operator.py:366-373 (recap/kernels/block_sparse.py:78-139).
 * Each query block walks its kept key blocks first, in the order the block-sparse pass
 * takes them, writes the head output and LSE, then walks the omitted blocks to the dense
 * result.  On the query blocks below dense_start (every row a refinement reads) the head
 * equals recap_block_sparse_fmha's (all_blocks = 0, out_pos NULL, the same k_norm_max) bit
 * for bit: the same kept blocks in the same order and the same arithmetic.  The dense query
 * blocks attend every key block in both, in an order that can differ (fp32 rounding).
 *   out / lse           [banks, S, D] bf16 / [banks, S] fp32 dense result, reordered row r at
 *                       row out_pos[r] (out_pos NULL: row r)
 *   head_out / head_lse [banks, S, D] bf16 / [banks, S] fp32 head result, reordered order */
int recap_refresh_attention(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                            const uint8_t* partition, const float* k_norm_max, int banks, int S, int D,
                            int n_video, float scale, const int32_t* out_pos, void* out, float* lse,
                            void* head_out, float* head_lse, int* status, void* stream);

/* recap_refresh_attention with the dense output written into the token shards of the ranks
 * of a sequence-parallel layer: bank b, native token n goes to out_ranks[q] + b out_bank_stride
 * + (n - q tokens_per_rank) out_row_stride (elements) with q = n / tokens_per_rank, straight
 * over NVLink for other GPUs (the head-to-sequence all-to-all after Operator.attend).
 * n_ranks in [2, 8], n_ranks * tokens_per_rank = S, strides multiples of 8, row stride >= D;
 * each out_ranks[q] 16-byte aligned.  The kernel ends with a system-scope fence; the caller
 * orders the ranks' reads of their shards after it (a collective on the stream). */
int recap_refresh_attention_ranks(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                                  const uint8_t* partition, const float* k_norm_max, int banks, int S, int D,
                                  int n_video, float scale, const int32_t* out_pos, void* const* out_ranks,
                                  int n_ranks, int tokens_per_rank, int64_t out_bank_stride, int64_t out_row_stride,
                                  float* lse, void* head_out, float* head_lse, int* status, void* stream);

/* The corrected SPARSE step: block-sparse attention with the drift-weighted merge of the coarse
 * tail and the cached refinement fused as its epilogue, written in native order.
 * Replaces block_sparse_exact + sparse_merge (recap/kernels/detail_cache.py:402-456) +
 * Layout.restore (recap/sparse/layout.py:92) of Operator._sparse (recap/operator.py:478-527).
 *   detail_value   [banks, rows, D] fp16, detail_log_mass/old_lse [banks, rows] fp32, center [banks]
 *   out            [banks, S, D] bf16, reordered row r at row out_pos[r]. */
int recap_sparse_step(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                      const uint8_t* partition, const float* k_norm_max, int banks, int S, int D, int n_video,
                      float scale,
                      const void* coarse_out, const float* coarse_lse, const void* detail_value,
                      const float* detail_log_mass, const float* old_lse, const float* center,
                      const int32_t* out_pos, void* out, int* status, void* stream);

/* recap_sparse_step with the output written into the token shards of the ranks of a
 * sequence-parallel layer, as recap_refresh_attention_ranks places it. */
int recap_sparse_step_ranks(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                            const uint8_t* partition, const float* k_norm_max, int banks, int S, int D, int n_video,
                            float scale, const void* coarse_out, const float* coarse_lse, const void* detail_value,
                            const float* detail_log_mass, const float* old_lse, const float* center,
                            const int32_t* out_pos, void* const* out_ranks, int n_ranks, int tokens_per_rank,
                            int64_t out_bank_stride, int64_t out_row_stride, int* status, void* stream);

/* Number of (err^2, ref^2) float pairs of scratch `partials` recap_refresh_detail needs. */
int recap_refresh_partials(int banks, int n_video);

/* Refinement write at a dense refresh, optionally scoring the old refinement first.
 * Replaces refresh_detail (recap/kernels/detail_cache.py:304-379).
 *   full_o/full_lse    dense output [banks, S, D] bf16 / [banks, S] fp32, native order
 *   head_o/head_lse    block-sparse output, reordered
 *   coarse_out/lse     [banks, rows, D] bf16 / [banks, rows]
 *   perm               [>= rows] int32 reordered video position -> native video index
 *   detail_value       [banks, rows, D] fp16 in/out; detail_log_mass [banks, rows] in/out
 *   validate           nonzero: stats[2] = (sum err^2, sum of^2) before the write
 *   old_lse/center     drift weight of the validation (both or neither; validate only). */
int recap_refresh_detail(const void* full_o, const float* full_lse, const void* head_o, const float* head_lse,
                         const void* coarse_out, const float* coarse_lse, const int32_t* perm, int banks, int S,
                         int D, int n_video, int video_offset, void* detail_value, float* detail_log_mass,
                         int validate, const float* old_lse, const float* center, float* partials,
                         float* stats, void* stream);

/* recap_refresh_detail without the `partials` scratch argument, for callers that may not
 * allocate device memory (hosts that pass a plugin only buffers they planned themselves,
 * or step loops that cannot afford the device synchronisation of cudaMalloc).  It has no
 * counterpart in the reference.  The validation partial sums live in a 1 MiB array inside
 * the library, held by every GPU that loads it until the process exits; the call rejects
 * problems with banks * ceil(rows / 32) > 131072 with RECAP_ERR_SCRATCH_LIMIT.  The first call on a
 * device looks the array's device address up (cudaGetSymbolAddress), so make that first
 * call before any stream capture.  All calls share the one array: calls that may overlap
 * on the GPU (different streams, or different host threads) race and must be ordered by
 * the caller.  Nothing in the array needs clearing: each call writes every entry it reads. */
int recap_refresh_detail_noalloc(const void* full_o, const float* full_lse, const void* head_o,
                                 const float* head_lse, const void* coarse_out, const float* coarse_lse,
                                 const int32_t* perm, int banks, int S, int D, int n_video, int video_offset,
                                 void* detail_value, float* detail_log_mass, int validate, const float* old_lse,
                                 const float* center, float* stats, void* stream);

/* Self-check of the polynomial exponential the attention softmax uses for part of
 * every row (2^y on the FP32 pipe, relative error below 1e-4 for -125 <= y <= 127;
 * y < -125 gives 2^-125 in place of zero): out[i] = 2^in[i] for n values.  No
 * counterpart in the reference; tests compare it with the CUDA exp2f of the same
 * inputs. */
int recap_exp2_check(const float* in, float* out, int n, void* stream);

/* Self-check of the bounded waits that every kernel of this library uses on its
 * on-chip barriers (no counterpart in the reference).  One thread waits on an
 * mbarrier that nothing arrives on until limit_ns (at most 1 s) runs out, writes
 * RECAP_STATUS_TIMEOUT_SELFTEST to *status and raises the block's abort flag; a second
 * waiter with a 4x longer limit leaves through that flag.  result[0], result[1]: 1 if
 * the first / second wait completed (expected 0); result[2]: the second waiter's time
 * in ns (about limit_ns, not 4x).  Nothing faults or hangs; the context stays usable. */
int recap_wait_selftest(int* status, long long limit_ns, long long* result, void* stream);

/* Buffers shared between the ranks of a sequence-parallel layer (one process per GPU), by CUDA
 * IPC: recap_peer_alloc allocates `bytes` on the current device (cudaMalloc), recap_peer_export
 * writes its recap_peer_handle_bytes()-byte handle, another process opens it with
 * recap_peer_import (peer access enabled on first use) and releases it with recap_peer_close;
 * the owner frees it with recap_peer_free after every importer has closed it.  No counterpart
 * in the reference: they carry the token shards recap_layout_gather_ranks reads and the
 * *_ranks attention passes write. */
int recap_peer_alloc(int64_t bytes, void** ptr);
int recap_peer_free(void* ptr);
int recap_peer_handle_bytes(void);
int recap_peer_export(void* ptr, void* handle_out);
int recap_peer_import(const void* handle, void** ptr);
int recap_peer_close(void* ptr);

/* The sequence-to-head exchange of a sequence-parallel layer as peer stores: rank `rank` of
 * n_ranks writes its projections src [tokens, 3, heads, D] bf16 (contiguous) into the receive
 * buffer of the rank owning each head group, recv_ranks[q] [n_ranks tokens, 3, heads / n_ranks,
 * D] (q's heads [q heads / n_ranks, (q + 1) heads / n_ranks)), at rows [rank tokens, (rank + 1)
 * tokens); other ranks' buffers opened with recap_peer_import, writes crossing NVLink.  The
 * caller orders the ranks around it (a collective on the stream before the owners read).  No
 * counterpart in the reference (it exchanges with all-to-all collectives). */
int recap_push_heads(const void* src, int tokens, int heads, int D, int rank, int n_ranks,
                     void* const* recv_ranks, void* stream);

/* Store a [banks, S, D] bf16 output (contiguous, 16-byte aligned) into the ranks' token shards
 * as the *_ranks attention passes place it (one kernel of 16-byte peer stores over NVLink):
 * the step after a REFRESH whose dense output the refinement write reads locally.  Strides
 * are multiples of 8 elements.  No counterpart in the reference. */
int recap_scatter_rows(const void* src, int banks, int S, int D, void* const* out_ranks, int n_ranks,
                       int tokens_per_rank, int64_t out_bank_stride, int64_t out_row_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RECAP_B200_H_ */
