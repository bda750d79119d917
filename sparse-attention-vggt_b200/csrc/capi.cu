// extern "C" entry points: argument validation and dispatch.
//
// Error behaviour mirrors the reference operator, which raises ValueError
// for unsupported dtypes (saf3r/triton/adaptive_block_attention.py:72-73):
// here every argument error returns a negative code and leaves a message in
// vggt_sparse_last_error(); nothing is launched in that case.
#include <cuda.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

thread_local char g_err[512] = "";

// limit of every pipeline wait in the tcgen05 attention kernels (0: the
// kernels' default of one second); see vggt_sparse_set_wait_limit_ns
std::atomic<uint64_t> g_wait_ns{0};
// see vggt_sparse_set_wait_selftest
std::atomic<int> g_wait_selftest{0};

int fail(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return -1;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int cuda_rc(cudaError_t e) {
  if (e == cudaSuccess) return 0;
  snprintf(g_err, sizeof(g_err), "CUDA error %d: %s", (int)e, cudaGetErrorString(e));
  return (int)e;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Multiprocessors of the current device (0 when it cannot be queried).
int current_device_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return sms;
}

// Splits per work item of the tcgen05 kernel: VGGT_ATTN_SPLIT (1-4) when set,
// else enough for about 8 waves of CTAs on the current device (1 for large
// grids).
int64_t attention_split(int64_t items) {
  if (const char* env = std::getenv("VGGT_ATTN_SPLIT")) {
    const long v = std::strtol(env, nullptr, 10);
    if (v >= 1 && v <= 4) return v;
  }
  return vggt::attn_tc05_split(items, current_device_sms());
}

// Index-row width (selected blocks per query block) below which a workspace
// call runs exactly the plain launch: with short selections the pairing's
// four launches and the key-range split cost more than they save (4 frames
// at top-k 25 %: 0.231 ms paired and split, 0.136 ms plain; 32 frames: 3.79
// against 4.08 ms).  VGGT_ATTN_PAIR_MIN overrides the default of 64.
int64_t pair_min_blocks() {
  if (const char* env = std::getenv("VGGT_ATTN_PAIR_MIN")) {
    const long v = std::strtol(env, nullptr, 10);
    if (v >= 0) return v;
  }
  return 64;
}

}  // namespace

extern "C" {

int vggt_sparse_version(void) { return (1 << 16) | 0; }

uint64_t vggt_sparse_set_wait_limit_ns(uint64_t ns) { return g_wait_ns.exchange(ns); }

int vggt_sparse_set_wait_selftest(int enable) {
  return g_wait_selftest.exchange(enable ? 1 : 0);
}

const char* vggt_sparse_last_error(void) { return g_err; }

size_t vggt_block_attention_workspace_size(int64_t n_tokens, int64_t n_patch, int64_t n_slots,
                                          int block_q, int block_k) {
  if (n_tokens <= 0 || n_patch <= 0 || n_slots <= 0 || block_q <= 0 || block_k <= 0) return 0;
  const int64_t qb = cdiv(n_tokens, block_q), nb = cdiv(n_patch, block_k);
  if (!vggt::qblock_pairing_supported(qb, nb)) return 0;
  // pair table, work order, the pairing scratch, then the split partials
  const int64_t items = n_slots * cdiv(qb, 2);
  return (((size_t)n_slots * cdiv(qb, 2) * 2 * 4 + 255) & ~(size_t)255) +
         (((size_t)n_slots * cdiv(qb, 2) * 4 + 255) & ~(size_t)255) +
         vggt::qblock_pairing_workspace(n_slots, qb, nb) +
         vggt::attn_tc05_split_bytes(items, attention_split(items));
}

int vggt_block_attention_ex(const void* q, const void* patch_k, const void* patch_v,
                            const void* special_k, const void* special_v, int dtype,
                            int64_t heads, int64_t n_tokens, int64_t n_patch, int64_t n_special,
                            int dim, const int32_t* indices, const int32_t* counts,
                            int counts_per_qblock, const int32_t* head_ids,
                            const uint8_t* head_dense, int64_t n_slots, int64_t max_blocks,
                            int block_q, int block_k, float scale, void* out, float* evidence,
                            int32_t* status, int kernel, void* stream, void* workspace,
                            size_t workspace_bytes) {
  g_err[0] = '\0';
  if (dtype != VGGT_DTYPE_BF16 && dtype != VGGT_DTYPE_FP16)
    return fail("Tensor-core sparse execution requires BF16 or FP16 (dtype code %d)", dtype);
  if (dim != 32 && dim != 64) return fail("head dim %d unsupported (32 or 64)", dim);
  if (block_q != 32 && block_q != 64) return fail("query_block %d unsupported (32, 64)", block_q);
  if (block_k != 32 && block_k != 64 && block_k != 128)
    return fail("key_block %d unsupported (32, 64, 128)", block_k);
  if (heads < 1 || n_tokens < 0 || n_patch < 0 || n_special < 0 || n_slots < 0 || max_blocks < 0)
    return fail("negative or empty size argument");
  if (n_slots > 65535) return fail("n_slots %lld exceeds 65535", (long long)n_slots);
  if (n_patch + n_special < 1 && n_tokens > 0 && n_slots > 0)
    return fail("no keys: n_patch + n_special must be >= 1");
  if (!std::isfinite(scale)) return fail("scale must be finite");
  if (kernel != VGGT_ATTN_AUTO && kernel != VGGT_ATTN_MMA_SYNC && kernel != VGGT_ATTN_TCGEN05)
    return fail("unknown kernel selector %d", kernel);
  if (n_slots == 0 || n_tokens == 0) return 0;
  if (!q || !patch_k || !patch_v || !out || !head_ids)
    return fail("q, patch_k, patch_v, out and head_ids must be non-NULL");
  if (n_special > 0 && (!special_k || !special_v))
    return fail("special_k/special_v must be non-NULL when n_special > 0");
  if (!counts || (max_blocks > 0 && !indices))
    return fail("indices and counts must be non-NULL");
  if (!aligned16(q) || !aligned16(patch_k) || !aligned16(patch_v) || !aligned16(out) ||
      (n_special > 0 && (!aligned16(special_k) || !aligned16(special_v))))
    return fail("q/k/v/out must be 16-byte aligned");

  vggt::AttnArgs a;
  a.q = q;
  a.pk = patch_k;
  a.pv = patch_v;
  a.sk = special_k ? special_k : patch_k;
  a.sv = special_v ? special_v : patch_v;
  a.out = out;
  a.indices = indices;
  a.counts = counts;
  a.head_ids = head_ids;
  a.head_dense = head_dense;
  a.evidence = evidence;
  a.status = status;
  a.heads = heads;
  a.n_tokens = n_tokens;
  a.n_patch = n_patch;
  a.n_special = n_special;
  a.n_slots = n_slots;
  a.max_blocks = max_blocks;
  a.qb_count = cdiv(n_tokens, block_q);
  a.nb = cdiv(n_patch, block_k);
  a.dim = dim;
  a.block_q = block_q;
  a.block_k = block_k;
  a.dtype = dtype;
  a.counts_per_qblock = counts_per_qblock ? 1 : 0;
  a.scale = scale;
  a.qblock_pairs = nullptr;
  a.work_order = nullptr;
  a.nsplit = 1;
  a.partial = nullptr;
  a.part_rows = nullptr;
  a.wait_ns = g_wait_ns.load();
  a.wait_selftest = g_wait_selftest.load();
  if (a.qb_count > 0x7fffffffLL) return fail("too many query blocks");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tc_ok = vggt::attn_tc05_supported(a);
  if (kernel == VGGT_ATTN_TCGEN05 && !tc_ok)
    return fail("tcgen05 kernel does not support this shape (needs dim 64, block_q 64, block_k 64)");
  if (kernel == VGGT_ATTN_TCGEN05 || (kernel == VGGT_ATTN_AUTO && tc_ok)) {
    const size_t need =
        vggt_block_attention_workspace_size(n_tokens, n_patch, n_slots, block_q, block_k);
    if (workspace != nullptr && need > 0 && max_blocks > 0 && max_blocks >= pair_min_blocks()) {
      if (workspace_bytes < need)
        return fail("workspace of %zu bytes, %zu needed", workspace_bytes, need);
      if (!aligned16(workspace)) return fail("workspace must be 16-byte aligned");
      // pair table first, then the work order, then the pairing scratch
      unsigned char* w = static_cast<unsigned char*>(workspace);
      int32_t* pairs = reinterpret_cast<int32_t*>(w);
      w += ((size_t)n_slots * cdiv(a.qb_count, 2) * 2 * 4 + 255) & ~(size_t)255;
      int32_t* order = reinterpret_cast<int32_t*>(w);
      w += ((size_t)n_slots * cdiv(a.qb_count, 2) * 4 + 255) & ~(size_t)255;
      const cudaError_t e = vggt::launch_qblock_pairing(indices, counts, a.counts_per_qblock,
                                                        head_dense, n_slots, a.qb_count,
                                                        max_blocks, a.nb, pairs, order, w, s);
      if (e != cudaSuccess) return cuda_rc(e);
      a.qblock_pairs = pairs;
      a.work_order = order;
      // split partials after the pairing scratch
      const int64_t items = n_slots * cdiv(a.qb_count, 2);
      const int64_t nsplit = attention_split(items);
      if (nsplit > 1) {
        unsigned char* sp = w + vggt::qblock_pairing_workspace(n_slots, a.qb_count, a.nb);
        a.nsplit = (int)nsplit;
        a.partial = reinterpret_cast<float*>(sp);
        a.part_rows = reinterpret_cast<int64_t*>(
            sp + (((size_t)items * nsplit * 66 * 128 * 4 + 255) & ~(size_t)255));
      }
    }
    return cuda_rc(vggt::launch_attn_tc05(a, s));
  }
  return cuda_rc(vggt::launch_attn_mma(a, s));
}

int vggt_block_attention(const void* q, const void* patch_k, const void* patch_v,
                         const void* special_k, const void* special_v, int dtype, int64_t heads,
                         int64_t n_tokens, int64_t n_patch, int64_t n_special, int dim,
                         const int32_t* indices, const int32_t* counts, int counts_per_qblock,
                         const int32_t* head_ids, const uint8_t* head_dense, int64_t n_slots,
                         int64_t max_blocks, int block_q, int block_k, float scale, void* out,
                         float* evidence, int32_t* status, int kernel, void* stream) {
  return vggt_block_attention_ex(q, patch_k, patch_v, special_k, special_v, dtype, heads,
                                 n_tokens, n_patch, n_special, dim, indices, counts,
                                 counts_per_qblock, head_ids, head_dense, n_slots, max_blocks,
                                 block_q, block_k, scale, out, evidence, status, kernel, stream,
                                 nullptr, 0);
}

int vggt_token_sparse_attention(const void* q, const void* k, const void* v,
                                const int32_t* indices, int64_t index_stride, int64_t n_queries,
                                int64_t n_keys, int64_t topk, int dim, int dtype, float scale,
                                void* out, int32_t* status, void* stream) {
  g_err[0] = '\0';
  if (dtype != VGGT_DTYPE_BF16 && dtype != VGGT_DTYPE_FP16)
    return fail("per-token sparse attention takes BF16 or FP16 (dtype code %d)", dtype);
  if (dim != 32 && dim != 64 && dim != 128) return fail("head dim %d unsupported (32, 64, 128)", dim);
  if (n_queries < 0 || n_keys < 0 || topk < 0 || index_stride < 0)
    return fail("negative size argument");
  if (!std::isfinite(scale)) return fail("scale must be finite");
  if (n_queries == 0) return 0;
  // one CTA per vggt::kTokenAttnQueriesPerCta queries; the grid's x extent is at most 2^31 - 1
  if (n_queries > (int64_t)0x7fffffff * vggt::kTokenAttnQueriesPerCta)
    return fail("too many queries (at most %lld)",
                (long long)0x7fffffff * vggt::kTokenAttnQueriesPerCta);
  if (!q || !k || !v || !out || (topk > 0 && !indices))
    return fail("q, k, v, out and indices must be non-NULL");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail("q/k/v/out must be 16-byte aligned");
  vggt::TokenAttnArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.indices = indices;
  a.index_stride = index_stride;
  a.n_queries = n_queries;
  a.n_keys = n_keys;
  a.topk = topk;
  a.dim = dim;
  a.dtype = dtype;
  a.scale = scale;
  a.out = out;
  a.status = status;
  return cuda_rc(vggt::launch_token_attention(a, static_cast<cudaStream_t>(stream)));
}

int vggt_frame_qk_topk(const void* q, const void* k, int32_t* out, int64_t batch,
                       int64_t n_queries, int64_t frames, int64_t tokens, int dim, int64_t topk,
                       int64_t groups, int32_t* status, void* stream) {
  g_err[0] = '\0';
  if (batch < 0 || n_queries < 0 || frames < 0 || tokens < 1 || topk < 1 || groups < 0)
    return fail("batch, n_queries, frames, groups must be >= 0 and tokens, topk >= 1");
  if (topk > tokens) topk = tokens;
  if (!vggt::frame_topk_supported(dim, topk))
    return fail("dim %d / topk %lld unsupported (dim 64 or 128, topk <= 128)", dim,
                (long long)topk);
  if (batch == 0 || n_queries == 0 || frames == 0) return 0;
  if (n_queries > 0x7fffffffLL || frames * tokens > 0x7fffffffLL || batch > 0x7fffffffLL)
    return fail("sizes above 2^31 rows are not supported");
  if (!q || !k || !out) return fail("q, k and out must be non-NULL");
  if (!aligned16(q) || !aligned16(k) || !aligned16(out))
    return fail("q/k/out must be 16-byte aligned");
  vggt::FrameTopkArgs a;
  a.q = q;
  a.k = k;
  a.out = out;
  a.status = status;
  a.batch = batch;
  a.n_queries = n_queries;
  a.frames = frames;
  a.tokens = tokens;
  a.topk = topk;
  a.dim = dim;
  a.groups = groups;
  return cuda_rc(vggt::launch_frame_topk(a, static_cast<cudaStream_t>(stream)));
}

int vggt_block_mask_assemble(const float* scores, int64_t n_slots, int64_t n_qblocks,
                             int64_t n_blocks, const int32_t* value_order, const int32_t* counts,
                             const int32_t* attention_counts, const int32_t* history,
                             int64_t history_len, int32_t* ids, uint8_t* origin,
                             int64_t max_blocks, int32_t* status, void* stream) {
  g_err[0] = '\0';
  if (n_slots < 0 || n_qblocks < 0 || n_blocks < 0 || history_len < 0 || max_blocks < 0)
    return fail("negative size argument");
  if (n_slots > 65535) return fail("n_slots %lld exceeds 65535", (long long)n_slots);
  if (n_slots == 0 || n_qblocks == 0) return 0;
  if (n_blocks < 1) return fail("n_blocks must be >= 1");
  if (history_len > 0x7fffffffLL) return fail("history_len too large");
  if (!vggt::assemble_supported(n_blocks))
    return fail("n_blocks %lld exceeds what one row's shared memory holds (about 50,000)",
                (long long)n_blocks);
  if (max_blocks < 1) return fail("max_blocks must be >= 1");
  if (!scores || !value_order || !counts || !attention_counts || !ids)
    return fail("scores, value_order, counts, attention_counts and ids must be non-NULL");
  if (history_len > 0 && !history) return fail("history must be non-NULL when history_len > 0");
  return cuda_rc(vggt::launch_assemble(scores, n_slots, n_qblocks, n_blocks, value_order, counts,
                                       attention_counts, history_len > 0 ? history : nullptr,
                                       history_len, ids, origin, max_blocks, status,
                                       static_cast<cudaStream_t>(stream)));
}

int vggt_history_update(const float* evidence, const int32_t* ids, int64_t n_slots,
                        int64_t n_qblocks, int64_t max_blocks, const int32_t* counts,
                        const int32_t* keeps, int32_t* new_history, int64_t history_len,
                        void* stream) {
  g_err[0] = '\0';
  if (n_slots < 0 || n_qblocks < 0 || max_blocks < 0 || history_len < 0)
    return fail("negative size argument");
  if (n_slots == 0 || n_qblocks == 0 || history_len == 0) return 0;
  if (max_blocks > 0x7fffffffLL) return fail("max_blocks too large");
  if (!evidence || !ids || !counts || !keeps || !new_history)
    return fail("evidence, ids, counts, keeps and new_history must be non-NULL");
  return cuda_rc(vggt::launch_history_update(evidence, ids, n_slots, n_qblocks, max_blocks, counts,
                                             keeps, new_history, history_len,
                                             static_cast<cudaStream_t>(stream)));
}

int vggt_block_mask_estimate(const void* q, const void* patch_k, int dtype, int64_t heads,
                             int64_t n_tokens, int64_t n_patch, int dim, const int32_t* head_ids,
                             int64_t n_slots, int block_q, int block_k, int mode, int64_t topk,
                             double tau, float scale, float* pooled_q, float* pooled_k,
                             int32_t* indices, int64_t max_blocks, int32_t* counts, float* scores,
                             int32_t* status, void* stream) {
  g_err[0] = '\0';
  if (dtype != VGGT_DTYPE_BF16 && dtype != VGGT_DTYPE_FP16)
    return fail("estimator requires BF16 or FP16 inputs (dtype code %d)", dtype);
  if (dim != 32 && dim != 64) return fail("head dim %d unsupported (32 or 64)", dim);
  if (block_q != 32 && block_q != 64 && block_q != 128)
    return fail("query_block %d unsupported (32, 64, 128)", block_q);
  if (block_k != 32 && block_k != 64 && block_k != 128)
    return fail("key_block %d unsupported (32, 64, 128)", block_k);
  if (heads < 1 || n_tokens < 0 || n_patch < 1 || n_slots < 0)
    return fail("invalid sizes (need heads >= 1, n_patch >= 1)");
  if (n_slots > 65535) return fail("n_slots %lld exceeds 65535", (long long)n_slots);
  if (!std::isfinite(scale)) return fail("scale must be finite");
  const int64_t qbc = cdiv(n_tokens, block_q), nb = cdiv(n_patch, block_k);
  if (nb > vggt::estimator_max_blocks_supported(dim))
    return fail("%lld key blocks exceed the supported maximum %d", (long long)nb,
                vggt::estimator_max_blocks_supported(dim));
  uint64_t tau_num = 0;
  if (mode == VGGT_SELECT_TOPK) {
    if (topk < 1) return fail("topk must be >= 1");
    if (max_blocks < std::min<int64_t>(topk, nb))
      return fail("max_blocks %lld < min(topk, n_blocks) = %lld", (long long)max_blocks,
                  (long long)std::min<int64_t>(topk, nb));
  } else if (mode == VGGT_SELECT_MASS) {
    if (!(tau > 0.0 && tau <= 1.0)) return fail("tau must be in (0, 1]");
    if (max_blocks < nb)
      return fail("max_blocks %lld < n_blocks %lld (mass selection may keep every block)",
                  (long long)max_blocks, (long long)nb);
    tau_num = (uint64_t)std::floor(tau * (double)(1ull << vggt::kTauBits) + 0.5);
    if (tau_num == 0) tau_num = 1;
  } else {
    return fail("unknown selection mode %d", mode);
  }
  if (n_slots == 0 || n_tokens == 0) return 0;
  if (!q || !patch_k || !head_ids || !pooled_q || !pooled_k || !indices || !counts)
    return fail("q, patch_k, head_ids, pooled_q, pooled_k, indices, counts must be non-NULL");
  if (!aligned16(q) || !aligned16(patch_k) || !aligned16(pooled_q) || !aligned16(pooled_k))
    return fail("q, patch_k and pooled scratch must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = cuda_rc(vggt::launch_pool(q, dtype, n_tokens, dim, block_q, qbc, head_ids, n_slots,
                                     heads, pooled_q, status, s));
  if (rc) return rc;
  rc = cuda_rc(vggt::launch_pool(patch_k, dtype, n_patch, dim, block_k, nb, head_ids, n_slots,
                                 heads, pooled_k, status, s));
  if (rc) return rc;
  return cuda_rc(vggt::launch_score_select(pooled_q, pooled_k, dim, qbc, nb, n_slots, scale, mode,
                                           topk, tau_num, indices, max_blocks, counts, scores, s));
}

size_t vggt_qkv_workspace_size(int64_t n_tokens, int heads) {
  if (n_tokens <= 0 || heads <= 0) return 0;
  return vggt::qkv_pool_partial_bytes(n_tokens, heads);
}

int vggt_qkv_project_pool(const void* x, const void* w_qkv, const void* b_qkv, int dtype,
                          int64_t n_tokens, int heads, int tokens_per_frame,
                          int special_per_frame, const float* q_norm_w, const float* q_norm_b,
                          const float* k_norm_w, const float* k_norm_b, float ln_eps,
                          const int32_t* pos, const float* rope_cos, const float* rope_sin,
                          int pos_count, void* q, void* patch_k, void* patch_v,
                          void* special_k, void* special_v, float* pooled_q, float* pooled_k,
                          void* workspace, size_t workspace_bytes, int32_t* status,
                          void* stream) {
  g_err[0] = '\0';
  if (dtype != VGGT_DTYPE_BF16 && dtype != VGGT_DTYPE_FP16)
    return fail("QKV projection takes BF16 or FP16 (dtype code %d)", dtype);
  if (heads < 1 || heads > 64) return fail("heads must be in [1, 64] (head dim 64)");
  if (n_tokens < 0) return fail("negative n_tokens");
  if (tokens_per_frame < 1 || special_per_frame < 0 || special_per_frame >= tokens_per_frame)
    return fail("need tokens_per_frame >= 1 and 0 <= special_per_frame < tokens_per_frame");
  if (n_tokens % tokens_per_frame != 0)
    return fail("n_tokens %lld is not a whole number of %d-token frames", (long long)n_tokens,
                tokens_per_frame);
  if (n_tokens > 0x7fffffffLL) return fail("n_tokens exceeds 2^31 - 1");
  if ((q_norm_w == nullptr) != (q_norm_b == nullptr) ||
      (k_norm_w == nullptr) != (k_norm_b == nullptr))
    return fail("LayerNorm weight and bias come together (both or neither)");
  if (!std::isfinite(ln_eps) || ln_eps < 0.f) return fail("ln_eps must be finite and >= 0");
  if (pos != nullptr && (rope_cos == nullptr || rope_sin == nullptr || pos_count < 1))
    return fail("RoPE needs rope_cos / rope_sin tables with pos_count >= 1");
  if (!vggt::qkv_pool_supported(pos != nullptr ? pos_count : 0))
    return fail("pos_count %d: the RoPE tables do not fit shared memory", pos_count);
  if (n_tokens == 0) return 0;
  if (!x || !w_qkv || !q || !patch_k || !patch_v ||
      (special_per_frame > 0 && (!special_k || !special_v)))
    return fail("x, w_qkv and the q / k / v outputs must be non-NULL");
  const int64_t c = (int64_t)heads * 64;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(x) || !a16(w_qkv) || !a16(q) || !a16(patch_k) || !a16(patch_v) ||
      (special_per_frame > 0 && (!a16(special_k) || !a16(special_v))) ||
      (b_qkv != nullptr && (reinterpret_cast<uintptr_t>(b_qkv) & 3u)))
    return fail("x, w_qkv and the outputs must be 16-byte aligned (bias 4-byte)");
  (void)c;
  const size_t need = vggt::qkv_pool_partial_bytes(n_tokens, heads);
  if (pooled_k != nullptr) {
    if (workspace == nullptr || workspace_bytes < need)
      return fail("pooled_k needs a workspace of %zu bytes", need);
    if (!a16(workspace)) return fail("workspace must be 16-byte aligned");
  }
  vggt::QkvPoolArgs a;
  a.x = x;
  a.w = w_qkv;
  a.bias = b_qkv;
  a.qn_w = q_norm_w;
  a.qn_b = q_norm_b;
  a.kn_w = k_norm_w;
  a.kn_b = k_norm_b;
  a.pos = pos;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.pos_count = pos_count;
  a.ln_eps = ln_eps;
  a.q = q;
  a.kp = patch_k;
  a.vp = patch_v;
  a.ks = special_k;
  a.vs = special_v;
  a.pooled_q = pooled_q;
  a.pooled_k = pooled_k;
  a.workspace = workspace;
  a.status = status;
  a.n_tokens = n_tokens;
  a.heads = heads;
  a.dtype = dtype;
  a.tok_per_frame = tokens_per_frame;
  a.special_per_frame = special_per_frame;
  return cuda_rc(vggt::launch_qkv_pool(a, static_cast<cudaStream_t>(stream)));
}

int vggt_block_select_pooled(const float* pooled_q, const float* pooled_k, int64_t pooled_heads,
                             const int32_t* head_ids, int64_t n_slots, int64_t n_qblocks,
                             int64_t n_blocks, int dim, int mode, int64_t topk, double tau,
                             float scale, int32_t* indices, int64_t max_blocks, int32_t* counts,
                             float* scores, int32_t* status, void* stream) {
  g_err[0] = '\0';
  if (dim != 32 && dim != 64) return fail("head dim %d unsupported (32 or 64)", dim);
  if (pooled_heads < 1 || n_slots < 0 || n_qblocks < 0 || n_blocks < 1)
    return fail("invalid sizes (need pooled_heads >= 1, n_blocks >= 1)");
  if (n_slots > 65535) return fail("n_slots %lld exceeds 65535", (long long)n_slots);
  if (!std::isfinite(scale)) return fail("scale must be finite");
  if (n_blocks > vggt::estimator_max_blocks_supported(dim))
    return fail("%lld key blocks exceed the supported maximum", (long long)n_blocks);
  uint64_t tau_num = 0;
  if (mode == VGGT_SELECT_TOPK) {
    if (topk < 1) return fail("topk must be >= 1");
    if (max_blocks < std::min<int64_t>(topk, n_blocks)) return fail("max_blocks too small");
  } else if (mode == VGGT_SELECT_MASS) {
    if (!(tau > 0.0 && tau <= 1.0)) return fail("tau must be in (0, 1]");
    if (max_blocks < n_blocks) return fail("max_blocks too small");
    tau_num = (uint64_t)std::floor(tau * (double)(1ull << vggt::kTauBits) + 0.5);
    if (tau_num == 0) tau_num = 1;
  } else {
    return fail("unknown selection mode %d", mode);
  }
  if (n_slots == 0 || n_qblocks == 0) return 0;
  if (!pooled_q || !pooled_k || !head_ids || !indices || !counts)
    return fail("pooled_q, pooled_k, head_ids, indices and counts must be non-NULL");
  return cuda_rc(vggt::launch_score_select_mapped(
      pooled_q, pooled_k, dim, n_qblocks, n_blocks, head_ids, pooled_heads, n_slots, scale, mode,
      topk, tau_num, indices, max_blocks, counts, scores, status,
      static_cast<cudaStream_t>(stream)));
}

int64_t vggt_kv_push_flag_bytes(int world) {
  if (world < 1 || world > vggt::kKvPushMaxPeers) return 0;
  return ((int64_t)(3 * world + 4) * 4 + 255) / 256 * 256;
}

int vggt_kv_push(const void* const* shards, const int64_t* rows_local,
                 const int64_t* dst_offsets, int n_tensors, int64_t heads, int dim,
                 int elem_bytes, void* const* rank_bases, int world, int rank,
                 int64_t flags_offset, int phase, uint32_t epoch, int handshake, int grid,
                 int32_t* status, void* stream) {
  g_err[0] = '\0';
  if (n_tensors < 1 || n_tensors > vggt::kKvPushMaxTensors)
    return fail("n_tensors must be in [1, %d]", vggt::kKvPushMaxTensors);
  if (world < 1 || world > vggt::kKvPushMaxPeers)
    return fail("world must be in [1, %d]", vggt::kKvPushMaxPeers);
  if (rank < 0 || rank >= world) return fail("rank %d outside [0, %d)", rank, world);
  if (phase != 0 && phase != 1) return fail("phase must be 0 or 1");
  if (heads < 0 || dim < 1 || (elem_bytes != 2 && elem_bytes != 4) ||
      ((int64_t)dim * elem_bytes) % 16)
    return fail("rows must be a multiple of 16 bytes (dim %d, %d-byte elements)", dim, elem_bytes);
  if (epoch == 0) return fail("epoch must be >= 1 (the flag words start at 0)");
  if (!shards || !rows_local || !dst_offsets || !rank_bases)
    return fail("shards, rows_local, dst_offsets and rank_bases must be non-NULL");
  if (flags_offset < 0 || flags_offset % 4) return fail("flags_offset must be a multiple of 4");
  vggt::KvPushArgs a{};
  a.n_tensors = n_tensors;
  a.row_units = (int64_t)dim * elem_bytes / 16;
  int64_t units = 0;
  for (int t = 0; t < n_tensors; ++t) {
    if (rows_local[t] < 1) return fail("rows_local[%d] must be >= 1", t);
    if (!shards[t] || !aligned16(shards[t])) return fail("shard %d must be 16-byte aligned", t);
    if (dst_offsets[t] < 0 || dst_offsets[t] % 16)
      return fail("dst_offsets[%d] must be a non-negative multiple of 16", t);
    a.src[t] = static_cast<const uint4*>(shards[t]);
    a.rows_local[t] = rows_local[t];
    a.dst_off[t] = dst_offsets[t];
    units += heads * rows_local[t] * a.row_units;
    a.unit_end[t] = units;
  }
  for (int j = 0; j < world; ++j) {
    if (!rank_bases[j] || !aligned16(rank_bases[j]))
      return fail("rank_bases[%d] must be a 16-byte aligned device address", j);
    a.peers[j] = rank_bases[j];
  }
  a.world = world;
  a.rank = rank;
  a.flags_off = flags_offset;
  a.phase = phase;
  a.epoch = epoch;
  a.handshake = handshake ? 1 : 0;
  a.status = status;
  const uint64_t lim = g_wait_ns.load();
  a.wait_ns = lim ? lim : 10000000000ull;  // ranks may start an exchange seconds apart
  if (grid <= 0) grid = std::max(1, current_device_sms());
  return cuda_rc(vggt::launch_kv_push(a, grid, static_cast<cudaStream_t>(stream)));
}

int vggt_block_select(const float* scores, int64_t rows, int64_t n_blocks, int mode, int64_t topk,
                      double tau, int32_t* indices, int64_t max_blocks, int32_t* counts,
                      void* stream) {
  g_err[0] = '\0';
  if (rows < 0 || n_blocks < 1) return fail("invalid sizes (need n_blocks >= 1)");
  if (n_blocks > vggt::estimator_max_blocks_supported(0))
    return fail("%lld blocks exceed the supported maximum", (long long)n_blocks);
  uint64_t tau_num = 0;
  if (mode == VGGT_SELECT_TOPK) {
    if (topk < 1) return fail("topk must be >= 1");
    if (max_blocks < std::min<int64_t>(topk, n_blocks)) return fail("max_blocks too small");
  } else if (mode == VGGT_SELECT_MASS) {
    if (!(tau > 0.0 && tau <= 1.0)) return fail("tau must be in (0, 1]");
    if (max_blocks < n_blocks) return fail("max_blocks too small");
    tau_num = (uint64_t)std::floor(tau * (double)(1ull << vggt::kTauBits) + 0.5);
    if (tau_num == 0) tau_num = 1;
  } else {
    return fail("unknown selection mode %d", mode);
  }
  if (rows == 0) return 0;
  if (!scores || !indices || !counts) return fail("scores, indices, counts must be non-NULL");
  return cuda_rc(vggt::launch_select_from_scores(scores, rows, n_blocks, mode, topk, tau_num,
                                                 indices, max_blocks, counts,
                                                 static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Estimator without caller-provided scratch.
//
// The estimator needs a temporary buffer for the pooled (block-mean) Q and K
// rows.  Some callers cannot hand one over: code running where no allocator
// may be called (inside a driver or plugin callback that forbids
// cudaMalloc, a runtime that pre-plans all device memory up front, or a
// host that is not allowed to grow GPU memory after start-up).  For them the
// pooled rows live in this fixed array in the library's own device memory.
// Every GPU that loads the library reserves it until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB of fp32 pooled rows
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
// Device address of the array per device ordinal, with the context it was
// looked up in: a device reset (or a released and re-created primary context)
// gives the array a new address, so a cached address is reused only while the
// same context is current.
struct NoallocCache {
  void* ctx;
  float* ptr;
};
NoallocCache g_noalloc_cache[kMaxDevices] = {};
std::mutex g_noalloc_mutex;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

// Device address of the scratch array on the current device.  The host-side
// name g_noalloc_scratch is only a stand-in for the symbol, never a device
// pointer, so the address is looked up with cudaGetSymbolAddress (with the
// device current) the first time a context uses it, then cached.
int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_rc(e);
  if (dev < 0 || dev >= kMaxDevices) return fail("device ordinal %d not supported", dev);
  CtxGetCurrentFn get = ctx_get_current_fn();
  if (get == nullptr) return fail("cuCtxGetCurrent is unavailable from the driver");
  CUcontext ctx = nullptr;  // stays null before the thread's first CUDA call
  if (get(&ctx) != CUDA_SUCCESS) return fail("cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoallocCache& c = g_noalloc_cache[dev];
  if (ctx == nullptr || c.ptr == nullptr || c.ctx != static_cast<void*>(ctx)) {
    void* ptr = nullptr;
    // also makes the device's primary context current when none was
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_rc(e);
    if (get(&ctx) != CUDA_SUCCESS || ctx == nullptr)
      return fail("no current CUDA context on device %d", dev);
    c.ctx = static_cast<void*>(ctx);
    c.ptr = static_cast<float*>(ptr);
  }
  *out = c.ptr;
  return 0;
}

}  // namespace

extern "C" int vggt_block_mask_estimate_noalloc(
    const void* q, const void* patch_k, int dtype, int64_t heads, int64_t n_tokens,
    int64_t n_patch, int dim, const int32_t* head_ids, int64_t n_slots, int block_q, int block_k,
    int mode, int64_t topk, double tau, float scale, int32_t* indices, int64_t max_blocks,
    int32_t* counts, float* scores, int32_t* status, void* stream) {
  g_err[0] = '\0';
  float* pooled_q = nullptr;
  float* pooled_k = nullptr;
  if (block_q > 0 && block_k > 0 && dim > 0 && n_tokens >= 0 && n_patch >= 0 && n_slots > 0 &&
      n_slots <= 65535) {
    const int64_t rows = cdiv(n_tokens, block_q) + cdiv(n_patch, block_k);
    const int64_t cap = (int64_t)(kNoAllocScratchBytes / sizeof(float));
    if (rows > cap / dim / n_slots)
      return fail("pooled rows need %lld bytes; the built-in scratch holds %lld bytes "
                  "(n_slots * (ceil(n_tokens/block_q) + ceil(n_patch/block_k)) * dim * 4)",
                  (long long)(n_slots * rows * dim * 4), (long long)kNoAllocScratchBytes);
    const int rc = noalloc_scratch(&pooled_q);
    if (rc) return rc;
    // both halves start on a 16-byte boundary: dim is a multiple of 32
    pooled_k = pooled_q + n_slots * cdiv(n_tokens, block_q) * dim;
  }
  // The pooling kernels write every pooled element they later read, so the
  // array's contents left by an earlier call never need clearing.
  return vggt_block_mask_estimate(q, patch_k, dtype, heads, n_tokens, n_patch, dim, head_ids,
                                  n_slots, block_q, block_k, mode, topk, tau, scale, pooled_q,
                                  pooled_k, indices, max_blocks, counts, scores, status, stream);
}
