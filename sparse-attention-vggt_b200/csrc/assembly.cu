// Device mask assembly with history and value order, and the same-pass
// history update.
//
// assemble: saf3r/patch/adaptive_block_value.py:42-91 (select_block_mask) for
// every (slot, query block) row at once.  Per row, one warp:
//   1. keys of the fp32 scores (monotone uint32) into shared memory;
//   2. with history and A >= 2: the cutoff is the score ranked min(nb, 2A);
//      of the history blocks, the A/2 (at most H) with the best current
//      scores are reused when they still score >= the cutoff;
//   3. the remaining A - |reused| attention slots take the best scores among
//      the blocks not yet taken;
//   4. the other count - A slots take the uncovered blocks in value order;
//   5. ascending ids with their origin (1 reused, 2 attention, 0 value).
// Every "best k" is one radix threshold over 4-bit digits with per-lane
// private histograms (unit weights) plus an in-order membership pass; ties go
// to the lower index (block id or history position).  The reference's
// torch.topk leaves that order unspecified.
//
// history update: :389-396 — per row, the `keep` ids whose same-pass
// evidence is largest among the first `count` slots, ascending (the
// reference keeps evidence order; later layers use the set).
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace vggt {

namespace assembly {

constexpr int RMAX = 8;  // rows (warps) per CTA at most

struct WarpHist {
  unsigned long long w[16][32];  // [digit][lane]
};

// Shared memory of one row (warp): its histogram (8-byte words), the keys and
// three bitmaps, rounded up to 16 bytes so the next warp's histogram stays
// aligned.
__host__ __device__ __forceinline__ size_t row_bytes(int64_t nb) {
  const int64_t nw = (nb + 31) / 32;
  return (sizeof(WarpHist) + (size_t)nb * 4 + (size_t)3 * nw * 4 + 15) & ~(size_t)15;
}

__device__ __forceinline__ bool bit_of(const uint32_t* bits, int i) {
  return (bits[i >> 5] >> (i & 31)) & 1u;
}

// Threshold of the k largest of n keys (key(i) for i < n): the k-th largest
// key `kth` and how many elements equal to it are taken (`ties`, the lowest
// indices first).  k == 0 selects nothing, k >= n everything.
template <class Key>
__device__ uint2 topk_threshold(int n, int64_t k, WarpHist* h, Key key) {
  const int lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  if (k <= 0) return make_uint2(0xffffffffu, 0u);
  if (k >= n) return make_uint2(0u, (uint32_t)n);
  uint32_t prefix = 0u, mask = 0u;
  unsigned long long above = 0ull;
  const unsigned long long target = (unsigned long long)k;
#pragma unroll 1
  for (int shift = 28; shift >= 0; shift -= 4) {
#pragma unroll
    for (int d = 0; d < 16; ++d) h->w[d][lane] = 0ull;
    for (int i = lane; i < n; i += 32) {
      const uint32_t kk = key(i);
      if ((kk & mask) == prefix) h->w[(kk >> shift) & 15u][lane] += 1ull;
    }
    __syncwarp();
    unsigned long long dsum = 0ull;
    if (lane < 16) {
#pragma unroll 8
      for (int l = 0; l < 32; ++l) dsum += h->w[lane][(l + lane) & 31];
    }
    unsigned long long suffix = dsum;
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) {
      const unsigned long long v = __shfl_down_sync(full, suffix, off);
      if (lane + off < 16) suffix += v;
    }
    const unsigned ball = __ballot_sync(full, lane < 16 && above + suffix >= target);
    const int digit = 31 - __clz(ball);
    above += __shfl_sync(full, suffix - dsum, digit);
    prefix |= (uint32_t)digit << shift;
    mask |= 15u << shift;
    __syncwarp();
  }
  return make_uint2(prefix, (uint32_t)(target - above));
}

// Calls act(i, in_set) for i = 0 .. n-1 in order, a warp chunk of 32 at a
// time (lane = i % 32), where in_set means key(i) is among the k largest.
template <class Key, class Act>
__device__ void for_each_member(int n, uint2 th, Key key, Act act) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  unsigned seen = 0u;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const bool valid = i < n;
    const uint32_t kk = valid ? key(i) : 0u;
    const bool gt = valid && kk > th.x;
    const bool eq = valid && kk == th.x;
    const unsigned eqb = __ballot_sync(0xffffffffu, eq);
    const bool in = gt || (eq && seen + __popc(eqb & lt) < th.y);
    act(base, i, valid, in);
    seen += __popc(eqb);
  }
}

__global__ void __launch_bounds__(RMAX * 32)
    assemble_kernel(const float* __restrict__ scores, int64_t qb_count, int nb,
                    const int32_t* __restrict__ value_order, const int32_t* __restrict__ counts,
                    const int32_t* __restrict__ attention_counts,
                    const int32_t* __restrict__ history, int hlen, int32_t* __restrict__ ids,
                    uint8_t* __restrict__ origin, int64_t max_blocks, int32_t* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  const unsigned lt = (1u << lane) - 1u;
  const int nw = (nb + 31) >> 5;
  unsigned char* mine = smem_raw + warp * row_bytes(nb);
  WarpHist* h = reinterpret_cast<WarpHist*>(mine);
  uint32_t* keys = reinterpret_cast<uint32_t*>(mine + sizeof(WarpHist));
  uint32_t* abits = keys + nb;   // attention (reused included)
  uint32_t* rbits = abits + nw;  // reused
  uint32_t* fbits = rbits + nw;  // value fill

  const int64_t slot = blockIdx.y;
  const int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (q >= qb_count) return;
  const int64_t row = slot * qb_count + q;
  const float* srow = scores + row * nb;
  int64_t count = counts[slot];
  count = count < 0 ? 0 : (count > nb ? nb : count);
  if (count > max_blocks) {
    if (lane == 0 && status) atomicOr(status, VGGT_STATUS_BAD_COUNT);
    count = max_blocks;
  }
  int64_t a_cnt = attention_counts[slot];
  a_cnt = a_cnt < 0 ? 0 : (a_cnt > count ? count : a_cnt);

  for (int i = lane; i < nb; i += 32) keys[i] = score_key(srow[i]);
  for (int i = lane; i < 3 * nw; i += 32) abits[i] = 0u;
  __syncwarp();

  if (a_cnt > 0) {
    const int32_t* hrow = history ? history + row * hlen : nullptr;
    if (hrow && hlen > 0 && a_cnt >= 2) {
      const int64_t eligible = a_cnt * 2 < nb ? a_cnt * 2 : nb;
      const uint2 cut = topk_threshold(nb, eligible, h, [&](int i) { return keys[i]; });
      // the eligible-th largest score's key: a history block is reused when
      // its current score reaches it
      const int64_t take = a_cnt / 2 < hlen ? a_cnt / 2 : hlen;
      auto hkey = [&](int j) -> uint32_t {
        const int b = hrow[j];
        return (b >= 0 && b < nb) ? keys[b] : 0u;  // invalid entries rank last
      };
      const uint2 th = topk_threshold(hlen, take, h, hkey);
      for_each_member(hlen, th, hkey, [&](int, int j, bool valid, bool in) {
        if (valid && in) {
          const int b = hrow[j];
          if (b >= 0 && b < nb && keys[b] >= cut.x) atomicOr(&rbits[b >> 5], 1u << (b & 31));
        }
      });
      __syncwarp();
      for (int i = lane; i < nw; i += 32) abits[i] = rbits[i];
      __syncwarp();
    }
    unsigned have = 0u;
    for (int i = lane; i < nw; i += 32) have += __popc(abits[i]);
    have = __reduce_add_sync(full, have);
    const int64_t remaining = a_cnt - (int64_t)have;
    if (remaining > 0) {
      auto k2 = [&](int i) -> uint32_t { return bit_of(abits, i) ? 0u : keys[i]; };
      const uint2 th = topk_threshold(nb, remaining, h, k2);
      for_each_member(nb, th, k2, [&](int base, int, bool, bool in) {
        const unsigned b = __ballot_sync(full, in);
        __syncwarp();  // every lane read its word before lane 0 updates it
        if (lane == 0 && b) abits[base >> 5] |= b;
      });
      __syncwarp();
    }
  }
  // value fill: the first count - A uncovered blocks in value order
  const int64_t quota = count - a_cnt;
  if (quota > 0) {
    int64_t run = 0;
    bool bad = false;
    for (int base = 0; base < nb && run < quota; base += 32) {
      const int p = base + lane;
      const int blk = p < nb ? value_order[p] : -1;
      const bool ok = blk >= 0 && blk < nb;
      bad |= p < nb && !ok;
      const bool v = ok && !bit_of(abits, blk);
      const unsigned vb = __ballot_sync(full, v);
      if (v && run + __popc(vb & lt) < quota) atomicOr(&fbits[blk >> 5], 1u << (blk & 31));
      run += __popc(vb);
    }
    if (__any_sync(full, bad) && lane == 0 && status) atomicOr(status, VGGT_STATUS_BAD_INDEX);
    __syncwarp();
  }
  // ascending ids with their origin
  int32_t* out = ids + row * max_blocks;
  uint8_t* org = origin ? origin + row * max_blocks : nullptr;
  int64_t written = 0;
  for (int base = 0; base < nb; base += 32) {
    const int i = base + lane;
    const bool sel = i < nb && (bit_of(abits, i) || bit_of(fbits, i));
    const unsigned sb = __ballot_sync(full, sel);
    const int64_t pos = written + __popc(sb & lt);
    if (sel && pos < max_blocks) {
      out[pos] = i;
      if (org) org[pos] = bit_of(rbits, i) ? 1 : (bit_of(abits, i) ? 2 : 0);
    }
    written += __popc(sb);
  }
  for (int64_t j = written + lane; j < max_blocks; j += 32) {
    out[j] = -1;
    if (org) org[j] = 0;
  }
}

// One warp per (slot, query block) row: the keep[slot] ids of the largest
// evidence among the first count[slot] slots, ascending (mask rows are
// ascending); -1 padded.
__global__ void __launch_bounds__(RMAX * 32)
    history_kernel(const float* __restrict__ evidence, const int32_t* __restrict__ ids,
                   int64_t rows_per_slot, int64_t n_rows, int64_t max_blocks,
                   const int32_t* __restrict__ counts, const int32_t* __restrict__ keeps,
                   int32_t* __restrict__ out, int64_t out_len) {
  __shared__ WarpHist hs[RMAX];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  const unsigned lt = (1u << lane) - 1u;
  const int64_t row = (int64_t)blockIdx.x * RMAX + warp;
  if (row >= n_rows) return;
  const int64_t slot = row / rows_per_slot;
  int64_t count = counts[slot];
  count = count < 0 ? 0 : (count > max_blocks ? max_blocks : count);
  int64_t keep = keeps[slot];
  keep = keep < 0 ? 0 : (keep > count ? count : (keep > out_len ? out_len : keep));
  const float* ev = evidence + row * max_blocks;
  const int32_t* id = ids + row * max_blocks;
  int32_t* dst = out + row * out_len;
  auto key = [&](int j) { return score_key(ev[j]); };
  const uint2 th = topk_threshold((int)count, keep, hs + warp, key);
  // mask rows hold ascending block ids, so the members in slot order are
  // already ascending
  int64_t written = 0;
  for_each_member((int)count, th, key, [&](int, int j, bool, bool in) {
    const unsigned b = __ballot_sync(full, in);
    if (in) dst[written + __popc(b & lt)] = id[j];
    written += __popc(b);
  });
  __syncwarp();
  for (int64_t j = written + lane; j < out_len; j += 32) dst[j] = -1;
}

}  // namespace assembly

bool assemble_supported(int64_t nb) { return assemble_smem_per_row(nb) <= kAssembleSmemBudget; }

size_t assemble_smem_per_row(int64_t nb) { return assembly::row_bytes(nb); }

cudaError_t launch_assemble(const float* scores, int64_t n_slots, int64_t qb_count, int64_t nb,
                            const int32_t* value_order, const int32_t* counts,
                            const int32_t* attention_counts, const int32_t* history,
                            int64_t hlen, int32_t* ids, uint8_t* origin, int64_t max_blocks,
                            int32_t* status, cudaStream_t stream) {
  using namespace assembly;
  if (n_slots == 0 || qb_count == 0) return cudaSuccess;
  // as many rows per CTA as fit in the shared-memory budget, up to RMAX
  int rows = (int)(kAssembleSmemBudget / assemble_smem_per_row(nb));
  rows = rows > RMAX ? RMAX : rows;
  if (rows < 1) return cudaErrorInvalidValue;
  const size_t smem = (size_t)rows * assemble_smem_per_row(nb);
  cudaError_t e = cudaFuncSetAttribute(assemble_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((qb_count + rows - 1) / rows), (unsigned)n_slots);
  assemble_kernel<<<grid, rows * 32, smem, stream>>>(scores, qb_count, (int)nb, value_order,
                                                    counts, attention_counts, history, (int)hlen,
                                                    ids, origin, max_blocks, status);
  return cudaGetLastError();
}

cudaError_t launch_history_update(const float* evidence, const int32_t* ids, int64_t n_slots,
                                  int64_t qb_count, int64_t max_blocks, const int32_t* counts,
                                  const int32_t* keeps, int32_t* out, int64_t out_len,
                                  cudaStream_t stream) {
  using namespace assembly;
  const int64_t rows = n_slots * qb_count;
  if (rows == 0) return cudaSuccess;
  history_kernel<<<(unsigned)((rows + RMAX - 1) / RMAX), RMAX * 32, 0, stream>>>(
      evidence, ids, qb_count, rows, max_blocks, counts, keeps, out, out_len);
  return cudaGetLastError();
}

}  // namespace vggt
