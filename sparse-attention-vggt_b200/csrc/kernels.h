// Internal launcher declarations shared by the C-ABI translation unit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vggt {

inline bool units_zero(int64_t a, int64_t b) { return a == 0 || b == 0; }

// estimator.cu
cudaError_t launch_pool(const void* x, int dtype, int64_t len, int d, int block, int64_t nblocks,
                        const int32_t* head_ids, int64_t n_slots, int64_t heads, float* pooled,
                        int32_t* status, cudaStream_t stream);
cudaError_t launch_score_select(const float* pq, const float* pk, int d, int64_t qb_count,
                                int64_t nb, int64_t n_slots, float scale, int mode, int64_t topk,
                                uint64_t tau_num, int32_t* indices, int64_t max_blocks,
                                int32_t* counts, float* scores_out, cudaStream_t stream);
// scores + selection from block means of every head: slot s reads head
// head_map[s] of [pooled_heads, ...] (out-of-range heads: BAD_HEAD, empty rows)
cudaError_t launch_score_select_mapped(const float* pq, const float* pk, int d, int64_t qb_count,
                                       int64_t nb, const int32_t* head_map, int64_t pooled_heads,
                                       int64_t n_slots, float scale, int mode, int64_t topk,
                                       uint64_t tau_num, int32_t* indices, int64_t max_blocks,
                                       int32_t* counts, float* scores_out, int32_t* status,
                                       cudaStream_t stream);
cudaError_t launch_select_from_scores(const float* scores, int64_t rows, int64_t nb, int mode,
                                      int64_t topk, uint64_t tau_num, int32_t* indices,
                                      int64_t max_blocks, int32_t* counts, cudaStream_t stream);
int estimator_max_blocks_supported(int d);

// Arguments of one block-sparse attention launch (device pointers).
struct AttnArgs {
  const void* q;
  const void* pk;
  const void* pv;
  const void* sk;
  const void* sv;
  void* out;
  const int32_t* indices;
  const int32_t* counts;
  const int32_t* head_ids;
  const uint8_t* head_dense;
  float* evidence;
  int32_t* status;
  // [n_indexed_slots, ceil(qb_count / 2), 2] query-block pairs of the
  // indexed slots (second entry -1 when alone), or null for (2p, 2p + 1)
  const int32_t* qblock_pairs;
  // [n_slots * ceil(qb_count / 2)] work items (slot * pairs + pair) in launch
  // order, or null for the natural order
  const int32_t* work_order;
  // tcgen05 only: each work item's tiles split over nsplit CTAs, merged by a
  // second launch; partial / part_rows sized by attn_tc05_split_bytes
  int nsplit;
  float* partial;
  int64_t* part_rows;
  int64_t heads, n_tokens, n_patch, n_special;
  int64_t n_slots, max_blocks, qb_count, nb;
  int dim, block_q, block_k, dtype, counts_per_qblock;
  float scale;
  // limit of every pipeline wait of the tcgen05 kernels (0: one second)
  uint64_t wait_ns;
  // nonzero: the tcgen05 kernel's MMA issuer first waits on a barrier that
  // nothing completes, so every CTA takes the timeout path (self-test)
  int wait_selftest;
};

// pairing.cu: query-block pairing for the 128-row tcgen05 tiles
constexpr int PAIR_WINDOW = 128;
size_t qblock_pairing_workspace(int64_t n_slots, int64_t qb_count, int64_t nb);
bool qblock_pairing_supported(int64_t qb_count, int64_t nb);
cudaError_t launch_qblock_pairing(const int32_t* indices, const int32_t* counts,
                                  int counts_per_qblock, const uint8_t* head_dense,
                                  int64_t n_slots, int64_t qb_count, int64_t max_blocks,
                                  int64_t nb, int32_t* pairs, int32_t* order, void* workspace,
                                  cudaStream_t stream);

// assembly.cu: select_block_mask with history and value order; history update
constexpr size_t kAssembleSmemBudget = 220 * 1024;
size_t assemble_smem_per_row(int64_t nb);
bool assemble_supported(int64_t nb);
cudaError_t launch_assemble(const float* scores, int64_t n_slots, int64_t qb_count, int64_t nb,
                            const int32_t* value_order, const int32_t* counts,
                            const int32_t* attention_counts, const int32_t* history,
                            int64_t hlen, int32_t* ids, uint8_t* origin, int64_t max_blocks,
                            int32_t* status, cudaStream_t stream);
cudaError_t launch_history_update(const float* evidence, const int32_t* ids, int64_t n_slots,
                                  int64_t qb_count, int64_t max_blocks, const int32_t* counts,
                                  const int32_t* keeps, int32_t* out, int64_t out_len,
                                  cudaStream_t stream);

// token_attention.cu: per-token sparse attention
struct TokenAttnArgs {
  const void* q;        // [n_queries, dim]
  const void* k;        // [n_keys, dim]
  const void* v;        // [n_keys, dim]
  const int32_t* indices;  // row r at indices + r * index_stride, topk entries
  int64_t index_stride, n_queries, n_keys, topk;
  int dim, dtype;
  float scale;
  void* out;            // [n_queries, dim]
  int32_t* status;
};
cudaError_t launch_token_attention(const TokenAttnArgs& a, cudaStream_t stream);
// queries handled by one CTA of the per-token kernel (one warp each)
constexpr int kTokenAttnQueriesPerCta = 4;

// frame_topk.cu: per-frame QK top-k
struct FrameTopkArgs {
  const void* q;       // [batch, n_queries, dim] bf16
  const void* k;       // [batch, frames * tokens, dim] bf16
  int32_t* out;        // [batch, n_queries, frames * topk]
  int32_t* status;
  int64_t batch, n_queries, frames, tokens, topk;
  int dim;
  int64_t groups;      // frame groups per query tile (0 = automatic)
};
bool frame_topk_supported(int dim, int64_t topk);
int64_t frame_topk_groups(int64_t frames, int64_t work_rows);
cudaError_t launch_frame_topk(const FrameTopkArgs& a, cudaStream_t stream);
// qkv_pool.cu: QKV projection + q/k LayerNorm + RoPE-2D + layout split + block means
struct QkvPoolArgs {
  const void* x;        // [n_tokens, heads * 64]
  const void* w;        // [3 * heads * 64, heads * 64] (nn.Linear weight)
  const void* bias;     // [3 * heads * 64] or null
  const float* qn_w;    // [64] or null
  const float* qn_b;
  const float* kn_w;
  const float* kn_b;
  const int32_t* pos;   // [n_tokens, 2] or null (no RoPE)
  const float* rope_cos;  // [pos_count, 16]
  const float* rope_sin;
  int pos_count;
  float ln_eps;
  void* q;              // [heads, n_tokens, 64]
  void* kp;
  void* vp;
  void* ks;
  void* vs;
  float* pooled_q;      // [heads, ceil(n_tokens / 64), 64] or null
  float* pooled_k;      // [heads, ceil(n_patch / 64), 64] or null
  void* workspace;      // qkv_pool_partial_bytes when pooled_k is set
  int32_t* status;
  int64_t n_tokens;
  int heads, dtype, tok_per_frame, special_per_frame;
};
size_t qkv_pool_partial_bytes(int64_t n_tokens, int heads);
bool qkv_pool_supported(int pos_count);
cudaError_t launch_qkv_pool(const QkvPoolArgs& a, cudaStream_t stream);
// attn_mma.cu
cudaError_t launch_attn_mma(const AttnArgs& a, cudaStream_t stream);
// attn_tc05.cu
bool attn_tc05_supported(const AttnArgs& a);
cudaError_t launch_attn_tc05(const AttnArgs& a, cudaStream_t stream);
// splits per work item for a grid of `items` 128-row work items on a device
// with `sms` multiprocessors, and the scratch bytes the split needs (0 when
// nsplit <= 1)
int64_t attn_tc05_split(int64_t items, int sms);
size_t attn_tc05_split_bytes(int64_t items, int64_t nsplit);
// merge launch of a key-range split (one CTA per work item)
cudaError_t launch_combine_splits(const AttnArgs& a, int64_t items, int nsplit,
                                  cudaStream_t stream);

// kv_push.cu: stores of this rank's frame shards into every rank's full
// buffers over peer memory (see the file's header for the flag protocol)
constexpr int kKvPushMaxPeers = 16;
constexpr int kKvPushMaxTensors = 4;
struct KvPushArgs {
  const uint4* src[kKvPushMaxTensors];    // shard t: [heads, rows_local[t], row_units] uint4
  int64_t rows_local[kKvPushMaxTensors];
  int64_t dst_off[kKvPushMaxTensors];     // byte offset of full tensor t in every allocation
  int64_t unit_end[kKvPushMaxTensors];    // cumulative 16-byte units of the shards
  int n_tensors;
  int64_t row_units;                      // 16-byte units per row
  void* peers[kKvPushMaxPeers];           // every rank's allocation base, rank order
  int world, rank;
  int64_t flags_off;                      // byte offset of the flag words
  int phase;                              // 0 or 1: which done/counter words
  uint32_t epoch;
  int handshake;
  int32_t* status;
  uint64_t wait_ns;
};
cudaError_t launch_kv_push(const KvPushArgs& a, int grid, cudaStream_t stream);

}  // namespace vggt
