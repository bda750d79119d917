/*
 * vggt_sparse.h — C ABI of the B200 (sm_100a) block-sparse global attention
 * used inside VGGT-style global-attention blocks.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), enqueues work on that stream, never synchronises and
 * never allocates: scratch buffers are caller-provided.  Return value 0 means
 * the work was enqueued; a negative value is an argument error (the message is
 * available from vggt_sparse_last_error()); a positive value is a CUDA error
 * code from the launch.
 *
 * Tensor layouts follow the reference operator
 * (saf3r/triton/adaptive_block_attention.py:63-83):
 *   q        [heads, n_tokens,  dim]   bf16 or fp16, contiguous
 *   patch_k  [heads, n_patch,   dim]   same dtype (patch tokens only)
 *   patch_v  [heads, n_patch,   dim]
 *   special_k[heads, n_special, dim]   camera + register tokens, always attended
 *   special_v[heads, n_special, dim]
 *   indices  [n_slots, ceil(n_tokens/block_q), max_blocks] int32, ascending
 *            unique patch-block ids; only the first `count` slots are read
 *   counts   [n_slots] int32 (reference) or [n_slots, n_qblocks] int32
 *   head_ids [n_slots] int32, the real head served by each slot
 *
 * Device-side validation: an index outside [0, ceil(n_patch/block_k)) or a
 * count outside [0, max_blocks] is never dereferenced; the kernel skips it and
 * ORs a VGGT_STATUS_* bit into *status (when status is non-NULL).
 */
#ifndef VGGT_SPARSE_H
#define VGGT_SPARSE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define VGGT_DTYPE_BF16 0
#define VGGT_DTYPE_FP16 1

/* selection modes of the block-mask estimator */
#define VGGT_SELECT_TOPK 0 /* k highest pooled scores, ties -> lower block id */
#define VGGT_SELECT_MASS 1 /* smallest prefix of the descending order whose softmax mass reaches tau */

/* attention kernel families */
#define VGGT_ATTN_AUTO 0    /* tcgen05 when the shape is supported, else the mma.sync kernel */
#define VGGT_ATTN_MMA_SYNC 1 /* warp-level mma.sync tiles, one CTA per (query block, slot) */
#define VGGT_ATTN_TCGEN05 2  /* TMA + tcgen05/TMEM kernel, 128-row tiles */

/* device status bits (ORed into *status) */
#define VGGT_STATUS_BAD_INDEX 1 /* a selected block id was outside [0, n_blocks) */
#define VGGT_STATUS_BAD_COUNT 2 /* a count was negative or above max_blocks */
#define VGGT_STATUS_TIMEOUT 4   /* a bounded pipeline wait expired; output is invalid */
#define VGGT_STATUS_BAD_HEAD 8  /* a head id was outside [0, heads); its rows were skipped */

/* Library version, (major << 16) | minor. */
int vggt_sparse_version(void);

/* Message of the last argument error on the calling thread ("" if none). */
const char* vggt_sparse_last_error(void);

/*
 * Failure detection.  No counterpart in the reference, whose Triton kernels
 * have no pipeline waits.  Every wait inside the tcgen05 attention kernels
 * (a TMA copy landing, an MMA finishing, a softmax warp publishing P) gives
 * up after this many nanoseconds; the launch then sets VGGT_STATUS_TIMEOUT,
 * lets its copies and MMAs in flight finish, releases its tensor memory and
 * returns, leaving the context usable (the output is invalid).  0 restores
 * the default of one second.  Process-wide; applies to launches enqueued
 * after the call.  Returns the previous setting.
 */
uint64_t vggt_sparse_set_wait_limit_ns(uint64_t ns);

/*
 * Self-test of the failure path above (no counterpart in the reference).
 * While enabled (nonzero), every tcgen05 attention launch first waits on a
 * barrier that nothing completes, so each of its CTAs runs out of its wait
 * limit and takes the abort path: VGGT_STATUS_TIMEOUT is set, nothing is
 * left in flight, the output is invalid and the context stays usable.  Meant
 * for tests, with a short wait limit.  Returns the previous setting.
 */
int vggt_sparse_set_wait_selftest(int enable);

/*
 * Block-sparse attention forward (with optional same-pass evidence).
 * Replaces saf3r/triton/adaptive_block_attention.py:63-83 (block_attention)
 * and its Triton kernel _forward (:7-60).
 *
 * head_dense  [n_slots] uint8 or NULL.  A slot whose flag is 1 attends to all
 *             patch blocks in order (no index reads) plus the specials: the
 *             dense path of the same kernel (head-profile dispatch).
 * counts_per_qblock  0: counts is [n_slots]; 1: counts is [n_slots, n_qblocks].
 * evidence    [n_slots, n_qblocks, max_blocks] fp32 or NULL.  When non-NULL,
 *             slot j of a query block receives the mean, over valid query
 *             rows, of the row log-sum-exp of that key block's logits
 *             (adaptive_block_attention.py:29-33).  Slots >= count are not
 *             written (callers pre-fill -inf).
 * out         [heads, n_tokens, dim], same dtype as q.  Only rows of the
 *             heads named in head_ids are written.
 * kernel      VGGT_ATTN_*.
 */
int vggt_block_attention(const void* q, const void* patch_k, const void* patch_v,
                         const void* special_k, const void* special_v, int dtype,
                         int64_t heads, int64_t n_tokens, int64_t n_patch, int64_t n_special,
                         int dim, const int32_t* indices, const int32_t* counts,
                         int counts_per_qblock, const int32_t* head_ids,
                         const uint8_t* head_dense, int64_t n_slots, int64_t max_blocks,
                         int block_q, int block_k, float scale, void* out, float* evidence,
                         int32_t* status, int kernel, void* stream);

/*
 * vggt_block_attention with a scheduling workspace.  No counterpart in the
 * reference (its Triton kernel runs one 64-row query block per program); the
 * arguments before `workspace` are those of vggt_block_attention.
 *
 * The tcgen05 kernel runs two query blocks per 128-row tile over the union of
 * their selections.  Given a workspace of at least
 * vggt_block_attention_workspace_size() bytes (16-byte aligned, device
 * memory), it first pairs the query blocks of every indexed slot so that the
 * two selections of a tile differ least (three small kernels on `stream`),
 * which removes most of the masked tile work; the output is bit-identical
 * to the unpaired run.  When the grid is small (fewer than 1,184 128-row
 * work items, e.g. one rank's query-block shard), the workspace also holds
 * partial results: each work item's key tiles are split over 2-4 CTAs and a
 * second launch merges them (output within rounding of the unsplit run; the
 * environment variable VGGT_ATTN_SPLIT=1..4 fixes the split, for both this
 * call and the size query).  workspace == NULL, a kernel choice other than
 * tcgen05, or short selections (max_blocks below 64, where the pairing and
 * the split cost more than they save; VGGT_ATTN_PAIR_MIN sets the threshold)
 * run exactly vggt_block_attention.  A workspace smaller than the
 * size query is an argument error.
 */
int vggt_block_attention_ex(const void* q, const void* patch_k, const void* patch_v,
                            const void* special_k, const void* special_v, int dtype,
                            int64_t heads, int64_t n_tokens, int64_t n_patch, int64_t n_special,
                            int dim, const int32_t* indices, const int32_t* counts,
                            int counts_per_qblock, const int32_t* head_ids,
                            const uint8_t* head_dense, int64_t n_slots, int64_t max_blocks,
                            int block_q, int block_k, float scale, void* out, float* evidence,
                            int32_t* status, int kernel, void* stream, void* workspace,
                            size_t workspace_bytes);

/* Workspace bytes vggt_block_attention_ex needs for query-block pairing (0 when
 * the shape is not paired: fewer than 2 query blocks, or more than 65536 key
 * blocks). */
size_t vggt_block_attention_workspace_size(int64_t n_tokens, int64_t n_patch, int64_t n_slots,
                                           int block_q, int block_k);

/*
 * Per-token sparse attention.  Replaces saf3r/triton/sparse_topk_attention.py:115-166
 * (fused_sparse_topk_attention) and :261-286 (fused_sparse_topk_attention_2,
 * its online-softmax form for top-k above 2048): each query attends to its
 * own key list, out[n] = softmax_j(q_n . k[idx[n, j]] * scale) . v[idx[n, j]],
 * fp32 softmax and accumulation, any topk.
 *
 * q            [n_queries, dim], k and v [n_keys, dim], out [n_queries, dim]:
 *              bf16 or fp16, contiguous, 16-byte aligned; dim 32, 64 or 128
 * indices      int32; query r's list starts at indices + r * index_stride
 *              (index_stride 0 = one list shared by every query, as the
 *              reference's stride-zero expanded view); duplicates count twice
 * Entries outside [0, n_keys) are skipped and set VGGT_STATUS_BAD_INDEX in
 * *status (the reference reads them unchecked); a query with no valid entry
 * gets zeros.
 */
int vggt_token_sparse_attention(const void* q, const void* k, const void* v,
                                const int32_t* indices, int64_t index_stride, int64_t n_queries,
                                int64_t n_keys, int64_t topk, int dim, int dtype, float scale,
                                void* out, int32_t* status, void* stream);

/*
 * Per-frame QK top-k.  Replaces saf3r/triton/fused_qk_topk.py:128-217
 * (compute_qk_topk_indices_fused) and its kernel _fused_perframe_qk_topk_kernel
 * (:24-108): for every query row and every frame of `tokens` consecutive keys,
 * the global indices of the frame's min(topk, tokens) largest scores q . k
 * (fp32 accumulation of the bf16 inputs, no scaling), in descending order,
 * ties to the lower key index; scores order as their sortable 32-bit keys
 * (the float order with +0 above -0).
 *
 * q      [batch, n_queries, dim] bf16, contiguous, 16-byte aligned
 * k      [batch, frames * tokens, dim] bf16, contiguous, 16-byte aligned
 * out    [batch, n_queries, frames * min(topk, tokens)] int32, 16-byte aligned;
 *        frame f's entries are keys f * tokens .. (f + 1) * tokens - 1
 * dim    64 or 128 (callers zero-pad other head dims: the scores are unchanged)
 * topk   1..128 after clamping to tokens
 * groups frame groups per 128-row query tile (0 = automatic)
 */
int vggt_frame_qk_topk(const void* q, const void* k, int32_t* out, int64_t batch,
                       int64_t n_queries, int64_t frames, int64_t tokens, int dim, int64_t topk,
                       int64_t groups, int32_t* status, void* stream);

/*
 * Mask assembly with history and value order.  Replaces
 * saf3r/patch/adaptive_block_value.py:42-91 (select_block_mask), run there per
 * head in Python, for every (slot, query block) row in one launch.
 *
 * scores            [n_slots, n_qblocks, n_blocks] fp32 relevance per key block
 * value_order       [n_blocks] int32, the value-coverage order of the blocks
 * counts            [n_slots] int32, blocks per row (the reference's `count`)
 * attention_counts  [n_slots] int32, attention-chosen blocks (`attention_count`)
 * history           [n_slots, n_qblocks, history_len] int32 block ids of the
 *                   previous layer, -1 where empty; NULL (or history_len 0) = none
 * ids               out [n_slots, n_qblocks, max_blocks] int32: ascending ids,
 *                   -1 padded
 * origin            out [n_slots, n_qblocks, max_blocks] uint8 or NULL:
 *                   1 reused from history, 2 attention, 0 value fill
 * With history and attention_count >= 2, up to attention_count / 2 history
 * blocks are reused when their current score ranks within the top
 * 2 * attention_count; the rest of the attention slots take the best current
 * scores; count - attention_count slots take uncovered blocks in value order.
 * Ties rank the lower block id (or history position) first; the reference's
 * torch.topk leaves their order unspecified.  n_blocks up to about 50,000.
 */
int vggt_block_mask_assemble(const float* scores, int64_t n_slots, int64_t n_qblocks,
                             int64_t n_blocks, const int32_t* value_order, const int32_t* counts,
                             const int32_t* attention_counts, const int32_t* history,
                             int64_t history_len, int32_t* ids, uint8_t* origin,
                             int64_t max_blocks, int32_t* status, void* stream);

/*
 * Same-pass history update.  Replaces adaptive_block_value.py:389-396
 * (winners = evidence.topk(keep); new_history = masks.gather(winners)).
 *
 * evidence     [n_slots, n_qblocks, max_blocks] fp32 (vggt_block_attention)
 * ids          [n_slots, n_qblocks, max_blocks] int32 ascending mask ids
 * counts/keeps [n_slots] int32: slots in use per row, history blocks to keep
 * new_history  out [n_slots, n_qblocks, history_len] int32: the keep ids of
 *              largest evidence (ties to the lower slot), ascending, -1 padded
 *              (the reference keeps evidence order; later layers use the set)
 */
int vggt_history_update(const float* evidence, const int32_t* ids, int64_t n_slots,
                        int64_t n_qblocks, int64_t max_blocks, const int32_t* counts,
                        const int32_t* keeps, int32_t* new_history, int64_t history_len,
                        void* stream);

/*
 * Block-mask estimator.  Mean-pools q over query blocks of block_q tokens and
 * patch_k over key blocks of block_k tokens (saf3r/patch/adaptive_block_value.py:16-23,
 * applied to both), forms pooled scores S = (Qbar . Kbar^T) * scale in fp32
 * (saf3r/patch/coarse_sensing.py:25-31), and selects key blocks per query
 * block: top-k (adaptive_block_value.py:54-56, ties -> lower id) or the
 * cumulative softmax-mass threshold tau (region_history_attention.py:39-42).
 * Special tokens are never pooled: the attention kernel always attends them.
 *
 * head_ids       [n_slots] int32: heads to estimate (the sparse heads).
 * pooled_q       caller scratch, fp32 [n_slots, ceil(n_tokens/block_q), dim]
 * pooled_k       caller scratch, fp32 [n_slots, ceil(n_patch/block_k), dim]
 * indices        out, int32 [n_slots, n_qblocks, max_blocks], ascending ids, -1 padded
 * counts         out, int32 [n_slots, n_qblocks]
 * scores         out or NULL, fp32 [n_slots, n_qblocks, n_blocks] pooled scores
 * topk           VGGT_SELECT_TOPK: blocks kept per row (clamped to n_blocks)
 * tau            VGGT_SELECT_MASS: mass threshold in (0, 1]
 * max_blocks     >= min(topk, n_blocks) for top-k; >= n_blocks for mass
 * status         device int32 or NULL; VGGT_STATUS_BAD_HEAD is ORed in for a
 *                head id outside [0, heads) (its pooled rows are zero)
 */
int vggt_block_mask_estimate(const void* q, const void* patch_k, int dtype, int64_t heads,
                             int64_t n_tokens, int64_t n_patch, int dim,
                             const int32_t* head_ids, int64_t n_slots, int block_q,
                             int block_k, int mode, int64_t topk, double tau, float scale,
                             float* pooled_q, float* pooled_k, int32_t* indices,
                             int64_t max_blocks, int32_t* counts, float* scores,
                             int32_t* status, void* stream);

/*
 * vggt_block_mask_estimate without the pooled_q / pooled_k scratch arguments.
 * No counterpart in the reference (it exists for callers of this C ABI that
 * cannot allocate device memory: code that runs where cudaMalloc is not
 * allowed, or whose device memory is planned once at start-up).  The pooled
 * rows go to a fixed 8 MiB array inside the library instead; every GPU that
 * loads the library holds that array until the process exits.
 *
 * Inputs, outputs and results are those of vggt_block_mask_estimate.  The
 * call allocates nothing.  It fails (negative return, message in
 * vggt_sparse_last_error) when
 *   n_slots * (ceil(n_tokens/block_q) + ceil(n_patch/block_k)) * dim * 4
 * exceeds 8 MiB (e.g. 16 heads x 43,968 tokens x 64 dims needs 5.6 MiB).
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  The address is cached per device together
 * with the CUDA context it belongs to; after cudaDeviceReset (or when the
 * primary context is released and created again) the next call sees a new
 * context and looks the address up again, so that call should also come
 * before any stream capture.  All calls share the one array: calls whose
 * work can overlap on the GPU (other streams, other threads) race on it and
 * must be serialised by the caller.
 */
int vggt_block_mask_estimate_noalloc(const void* q, const void* patch_k, int dtype, int64_t heads,
                                     int64_t n_tokens, int64_t n_patch, int dim,
                                     const int32_t* head_ids, int64_t n_slots, int block_q,
                                     int block_k, int mode, int64_t topk, double tau, float scale,
                                     int32_t* indices, int64_t max_blocks, int32_t* counts,
                                     float* scores, int32_t* status, void* stream);

/*
 * QKV projection with the estimator's pooling fused into its epilogue.
 * Replaces the steps of saf3r/patch/adaptive_block_value.py:297-315 before
 * the estimator: the `qkv` Linear (x [n_tokens, C] times w_qkv [3C, C]^T plus
 * b_qkv [3C], C = 64 * heads, output rounded to the input dtype), q_norm /
 * k_norm (LayerNorm over each head's 64 dims with weight / bias [64] fp32 and
 * ln_eps; NULL for none), RoPE-2D of q and k (saf3r/models/official_vggt/
 * layers/rope.py; pos [n_tokens, 2] int32 (y, x) and cos / sin tables
 * [pos_count, 16] fp32 of position * base^(-i/16); pos NULL for none), the
 * token layout's split (tokens_per_frame tokens per frame, the first
 * special_per_frame of each special) into q [heads, n_tokens, 64],
 * patch_k / patch_v [heads, n_patch, 64], special_k / special_v
 * [heads, n_special, 64], and the estimator's block means
 * (adaptive_block_value.py:16-23): pooled_q [heads, ceil(n_tokens/64), 64] and
 * pooled_k [heads, ceil(n_patch/64), 64] fp32 (either may be NULL; pooled_k
 * needs a workspace of vggt_qkv_workspace_size() bytes).  The means are
 * computed in a fixed order (deterministic).
 */
size_t vggt_qkv_workspace_size(int64_t n_tokens, int heads);
int vggt_qkv_project_pool(const void* x, const void* w_qkv, const void* b_qkv, int dtype,
                          int64_t n_tokens, int heads, int tokens_per_frame,
                          int special_per_frame, const float* q_norm_w, const float* q_norm_b,
                          const float* k_norm_w, const float* k_norm_b, float ln_eps,
                          const int32_t* pos, const float* rope_cos, const float* rope_sin,
                          int pos_count, void* q, void* patch_k, void* patch_v,
                          void* special_k, void* special_v, float* pooled_q, float* pooled_k,
                          void* workspace, size_t workspace_bytes, int32_t* status,
                          void* stream);

/*
 * Scores + selection from block means of every head (e.g. the output of
 * vggt_qkv_project_pool): slot s uses head head_ids[s] of pooled_q
 * [pooled_heads, n_qblocks, dim] and pooled_k [pooled_heads, n_blocks, dim].
 * Outputs and rules are those of vggt_block_mask_estimate.  A head id
 * outside [0, pooled_heads) leaves its rows empty and sets
 * VGGT_STATUS_BAD_HEAD.
 */
int vggt_block_select_pooled(const float* pooled_q, const float* pooled_k, int64_t pooled_heads,
                             const int32_t* head_ids, int64_t n_slots, int64_t n_qblocks,
                             int64_t n_blocks, int dim, int mode, int64_t topk, double tau,
                             float scale, int32_t* indices, int64_t max_blocks, int32_t* counts,
                             float* scores, int32_t* status, void* stream);

/*
 * Selection only, from caller-supplied fp32 pooled scores [rows, n_blocks]
 * (row-major).  Used to re-run the selection rule on exported scores.
 */
int vggt_block_select(const float* scores, int64_t rows, int64_t n_blocks, int mode,
                      int64_t topk, double tau, int32_t* indices, int64_t max_blocks,
                      int32_t* counts, void* stream);

/*
 * No reference counterpart (the reference runs on one GPU): the K/V exchange
 * of the sequence-parallel layer over NVLink peer memory.  Every rank keeps
 * its full head-major K/V buffers in one allocation of the same size and
 * layout on every rank, mapped into every other rank's address space
 * (rank_bases[j] = rank j's allocation as this process addresses it), with
 * vggt_kv_push_flag_bytes(world) bytes of flag words at flags_offset
 * (zeroed once before the first exchange).  The launch stores this rank's
 * shard t ([heads, rows_local[t], dim], contiguous) into rows
 * [rank * rows_local[t], (rank + 1) * rows_local[t]) of every head of full
 * tensor t ([heads, world * rows_local[t], dim] at byte dst_offsets[t] of
 * every allocation), and completes once this rank's full buffers hold every
 * rank's rows.  Every rank makes the same calls in the same order with the
 * same epoch (>= 1, raised by one per exchange); handshake = 1 on the first
 * call of an exchange makes every rank wait until all ranks have started it
 * (their previous readers of the buffers are done), phase 0/1 tells two
 * calls of one exchange apart.  Nothing reads another GPU's memory.  Waits
 * are bounded (vggt_sparse_set_wait_limit_ns, else 10 s); on expiry
 * VGGT_STATUS_TIMEOUT is ORed into *status and the buffers are invalid.
 * grid <= 0 picks one CTA per multiprocessor.
 */
int vggt_kv_push(const void* const* shards, const int64_t* rows_local,
                 const int64_t* dst_offsets, int n_tensors, int64_t heads, int dim,
                 int elem_bytes, void* const* rank_bases, int world, int rank,
                 int64_t flags_offset, int phase, uint32_t epoch, int handshake, int grid,
                 int32_t* status, void* stream);

/* Bytes of flag words vggt_kv_push needs for `world` ranks (0 if unsupported). */
int64_t vggt_kv_push_flag_bytes(int world);

#ifdef __cplusplus
}
#endif

#endif /* VGGT_SPARSE_H */
