// Block-mask estimator: mean pooling of Q / patch-K per block, fp32 pooled
// scores, and per-row selection (top-k or cumulative softmax mass).
//
// Reference behaviour restated here:
//   pooling    saf3r/patch/adaptive_block_value.py:16-23 (block_mean; the last
//              block divides by its real population)
//   scores     saf3r/patch/coarse_sensing.py:25-31 (fp32 Q . Kbar^T * scale)
//   top-k      saf3r/patch/adaptive_block_value.py:54-56 (topk, ids sorted);
//              ties broken toward the lower block id as in
//              saf3r/triton/fused_qk_topk.py:73-80
//   mass       saf3r/patch/region_history_attention.py:39-42 (sort descending,
//              cumsum, m = #(cumsum < tau) + 1, clamped to the row length)
//
// Both selection rules are one radix select over the monotone uint32 key of
// the fp32 score: each of four 8-bit passes histograms (count, weight) of the
// candidates sharing the decided prefix and keeps the highest digit whose
// suffix weight still reaches the target.  Top-k uses unit weights and target
// k; mass uses integer-quantised softmax weights (common.cuh) and target
// ceil(tau * W).  Sums are exact integers, so the result does not depend on
// summation order and the numpy oracle reproduces it bit for bit.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace vggt {

// ---------------------------------------------------------------------------
// Pooling: one warp per (slot, block).  16-byte vector loads; each lane keeps
// 8 fp32 column sums over the rows of its row group, then the row groups are
// folded with shuffles in a fixed order.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) pool_blocks_kernel(const T* __restrict__ x, int64_t len,
                                                          int block, int64_t nblocks,
                                                          const int32_t* __restrict__ head_ids,
                                                          int64_t n_slots, int64_t heads,
                                                          float* __restrict__ pooled,
                                                          int32_t* __restrict__ status) {
  constexpr int CH = D / 8;       // 16-byte chunks per row
  constexpr int RG = 32 / CH;     // row groups per warp
  const int lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (unit >= n_slots * nblocks) return;
  const int64_t slot = unit / nblocks;
  const int64_t blk = unit - slot * nblocks;
  const int64_t head = head_ids[slot];
  const int chunk = lane % CH;
  if (head < 0 || head >= heads) {
    if (lane == 0 && status) atomicOr(status, VGGT_STATUS_BAD_HEAD);
    if (lane < CH) {
      float4* dst = reinterpret_cast<float4*>(pooled + unit * D + lane * 8);
      dst[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      dst[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }
  const int rg = lane / CH;
  const int64_t row0 = blk * block;
  const int64_t rows = min((int64_t)block, len - row0);
  const uint4* src = reinterpret_cast<const uint4*>(x + (head * len + row0) * D) + chunk;

  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  // up to 128 rows per block -> at most 32 iterations per lane
#pragma unroll 4
  for (int r = rg; r < rows; r += RG) {
    uint4 v = __ldg(src + (int64_t)r * CH);
    float2 a = ElemOps<T>::to_float2(v.x);
    float2 b = ElemOps<T>::to_float2(v.y);
    float2 c = ElemOps<T>::to_float2(v.z);
    float2 d = ElemOps<T>::to_float2(v.w);
    acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
    acc[4] += c.x; acc[5] += c.y; acc[6] += d.x; acc[7] += d.y;
  }
#pragma unroll
  for (int off = CH; off < 32; off <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], off);
  }
  if (rg == 0) {
    const float pop = (float)rows;
    float4* dst = reinterpret_cast<float4*>(pooled + unit * D + chunk * 8);
    dst[0] = make_float4(acc[0] / pop, acc[1] / pop, acc[2] / pop, acc[3] / pop);
    dst[1] = make_float4(acc[4] / pop, acc[5] / pop, acc[6] / pop, acc[7] / pop);
  }
}

// ---------------------------------------------------------------------------
// Radix select of one row by one warp.
// ---------------------------------------------------------------------------
// 4-bit digits, eight passes from the top.  Each lane accumulates the weights
// (top-k: counts) of its own elements in a private column of the histogram,
// laid out [digit][lane] so that the 32 lanes hit 32 different 8-byte words:
// no atomics, no contention even when every key of the row shares its top
// digits (an fp32 key's top bits are its sign and exponent).
// Candidate ids are also kept, once they fit, in a per-warp list (uint16) so
// the remaining passes touch only them.
constexpr int kCandCap = 512;
struct SelectHist {
  unsigned long long w[16][32];
  uint16_t cand[kCandCap];
};

__device__ __forceinline__ uint32_t key_to_bits(uint32_t key) {
  return (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
}

// Selects one row of fp32 scores held in shared memory.  The row is
// overwritten with the monotone uint32 keys of its scores; mass weights are
// recomputed from the keys (exactly: a key maps back to its canonical score)
// for the elements still in the candidate range.  Writes ascending selected
// ids (and -1 padding) to out[0:max_blocks]; returns their count m.
__device__ int select_row_warp(float* __restrict__ srow, int nb, int mode, int64_t topk,
                               uint64_t tau_num, SelectHist* hist, int32_t* __restrict__ out,
                               int64_t max_blocks) {
  const int lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  const unsigned lt_mask = (1u << lane) - 1u;
  uint32_t* keys = reinterpret_cast<uint32_t*>(srow);
  const bool mass = mode == VGGT_SELECT_MASS;
  float rowmax = -INFINITY;
  uint64_t target, total;
  if (mass) {
    for (int i = lane; i < nb; i += 32) rowmax = fmaxf(rowmax, srow[i]);
#pragma unroll
    for (int off = 16; off; off >>= 1) rowmax = fmaxf(rowmax, __shfl_xor_sync(full, rowmax, off));
  }
  // keys once per element; the AND and OR of all keys give the leading bits
  // every key shares
  uint32_t kand = 0xffffffffu, kor = 0u;
  for (int i = lane; i < nb; i += 32) {
    const uint32_t key = score_key(srow[i]);
    keys[i] = key;
    kand &= key;
    kor |= key;
  }
  kand = __reduce_and_sync(full, kand);
  kor = __reduce_or_sync(full, kor);
  // top-k: total and target now; mass: the total weight W comes out of the
  // first radix pass, which sees every element, and then T = ceil(tau W)
  total = (uint64_t)nb;
  target = (uint64_t)(topk < (int64_t)nb ? topk : (int64_t)nb);
  __syncwarp();

  int m = -1;
  uint32_t prefix = 0u, prefix_mask = 0u;
  unsigned long long above_w = 0;
  // Every block is kept when k >= nb, or when no prefix reaches the mass target
  // (m = #(cum < T) + 1 then exceeds nb and is clamped).  A mass target equal to
  // the total still goes through the radix path: trailing zero-weight blocks
  // are excluded exactly as the reference's cumsum would exclude them.
  if (!mass && target == total) {
    m = nb;
  } else {
    // leading bits shared by every key are already decided: start at the
    // 4-bit digit holding the highest differing bit
    const uint32_t diff = kand ^ kor;
    const int top = diff ? 31 - __clz(diff) : 0;
    const int first = (top / 4) * 4;
    prefix_mask = first >= 28 ? 0u : (0xffffffffu << (first + 4));
    prefix = kand & prefix_mask;
    int ncand = -1;  // length of hist->cand, -1 while the candidates do not fit
#pragma unroll 1
    for (int shift = first; shift >= 0; shift -= 4) {
#pragma unroll
      for (int d = 0; d < 16; ++d) hist->w[d][lane] = 0ull;
      const int nscan = ncand < 0 ? nb : ncand;
      for (int j = lane; j < nscan; j += 32) {
        const int i = ncand < 0 ? j : (int)hist->cand[j];
        const uint32_t key = keys[i];
        if ((key & prefix_mask) == prefix) {
          const unsigned long long w =
              mass ? det_mass_weight(__uint_as_float(key_to_bits(key)), rowmax) : 1ull;
          hist->w[(key >> shift) & 15u][lane] += w;
        }
      }
      __syncwarp();
      // lane d < 16 totals digit d; the chosen digit is the highest one whose
      // suffix weight (plus everything already above the prefix) reaches the
      // target
      unsigned long long dsum = 0;
      if (lane < 16) {
        // skewed columns: the 16 lanes read 16 different banks
#pragma unroll 8
        for (int l = 0; l < 32; ++l) dsum += hist->w[lane][(l + lane) & 31];
      }
      unsigned long long suffix = dsum;
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) {
        const unsigned long long v = __shfl_down_sync(full, suffix, off);
        if (lane + off < 16) suffix += v;
      }
      if (mass && shift == first) {
        // every element is a candidate in the first pass: digit 0's suffix is W
        total = __shfl_sync(full, suffix, 0);
        target = mass_target(total, tau_num);
        if (target > total) {
          m = nb;
          break;
        }
      }
      const unsigned ball = __ballot_sync(full, lane < 16 && above_w + suffix >= target);
      const int digit = 31 - __clz(ball);
      above_w += __shfl_sync(full, suffix - dsum, digit);
      prefix |= (uint32_t)digit << shift;
      prefix_mask |= 15u << shift;
      __syncwarp();
      // (re)build the candidate list for the next pass: ids whose key matches
      // the longer prefix, in id order; abandoned when more than kCandCap match
      if (shift > 0) {
        const int nsrc = ncand < 0 ? nb : ncand;
        int written = 0;
        for (int base = 0; base < nsrc && written <= kCandCap; base += 32) {
          const int j = base + lane;
          int i = 0;
          bool keep = false;
          if (j < nsrc) {
            i = ncand < 0 ? j : (int)hist->cand[j];
            keep = (keys[i] & prefix_mask) == prefix;
          }
          const unsigned kb = __ballot_sync(full, keep);
          __syncwarp();  // every lane has read its source entry before any write
          const int pos = written + __popc(kb & lt_mask);
          if (keep && pos < kCandCap) hist->cand[pos] = (uint16_t)i;
          written += __popc(kb);
        }
        ncand = written <= kCandCap ? written : -1;
        __syncwarp();
        if (ncand >= 0 && ncand <= 32) {
          // Few candidates left (typically after three passes): settle the
          // remaining digits at once, one candidate per lane.  The remaining
          // passes would end on the largest candidate key K with
          // above + W(candidates with key >= K) >= target; the weight of the
          // candidates above K then joins `above`.  Same integer weights, so
          // the same selection.
          const bool have = lane < ncand;
          const uint32_t key = have ? keys[hist->cand[lane]] : 0u;
          const unsigned long long w =
              !have ? 0ull
                    : (mass ? det_mass_weight(__uint_as_float(key_to_bits(key)), rowmax) : 1ull);
          unsigned long long ge = 0ull;
          for (int j = 0; j < ncand; ++j) {
            const uint32_t kj = __shfl_sync(full, key, j);
            const unsigned long long wj = __shfl_sync(full, w, j);
            if (kj >= key) ge += wj;
          }
          const uint32_t kb = __reduce_max_sync(full, (have && above_w + ge >= target) ? key : 0u);
          unsigned long long gt = (have && key > kb) ? w : 0ull;
#pragma unroll
          for (int off = 16; off; off >>= 1) gt += __shfl_xor_sync(full, gt, off);
          above_w += gt;
          prefix = kb;
          prefix_mask = 0xffffffffu;
          break;
        }
      }
    }
  }
  if (m == nb) {
    for (int i = lane; i < nb; i += 32)
      if (i < max_blocks) out[i] = i;
  } else {
    // prefix is now the key of the last selected element; take enough of its
    // ties (lowest ids first) to reach the target
    unsigned long long tie_w = 1ull;
    if (mass) tie_w = det_mass_weight(__uint_as_float(key_to_bits(prefix)), rowmax);
    const unsigned long long need = target - above_w;  // > 0
    const unsigned int ties_taken = (unsigned int)((need + tie_w - 1ull) / tie_w);
    // compaction in id order; m is the number written
    unsigned int tie_seen = 0, written = 0;
    for (int base = 0; base < nb; base += 32) {
      const int i = base + lane;
      const bool valid = i < nb;
      const uint32_t key = valid ? keys[i] : 0u;
      const bool gt = valid && key > prefix;
      const bool eq = valid && key == prefix;
      const unsigned eqb = __ballot_sync(full, eq);
      const unsigned rank = tie_seen + __popc(eqb & lt_mask);
      const bool inc = gt || (eq && rank < ties_taken);
      const unsigned incb = __ballot_sync(full, inc);
      const unsigned pos = written + __popc(incb & lt_mask);
      if (inc && pos < max_blocks) out[pos] = i;
      written += __popc(incb);
      tie_seen += __popc(eqb);
    }
    m = (int)written;
  }
  for (int64_t j = m + lane; j < max_blocks; j += 32) out[j] = -1;
  return m;
}

// ---------------------------------------------------------------------------
// Scores + selection.  One CTA holds R query blocks of one slot: their pooled
// Q rows and their complete fp32 score rows live in shared memory; pooled K
// is streamed once per CTA.  Warps then select rows independently.
// ---------------------------------------------------------------------------
template <int D, bool FROM_SCORES, int RMAX>
__global__ void __launch_bounds__(256, 3) score_select_kernel(
    const float* __restrict__ pooled_q, const float* __restrict__ pooled_k, int64_t qb_count,
    int64_t nb, float scale, int mode, int64_t topk, uint64_t tau_num,
    int32_t* __restrict__ indices, int64_t max_blocks, int32_t* __restrict__ counts,
    float* __restrict__ scores_out, const float* __restrict__ scores_in,
    const int32_t* __restrict__ head_map, int64_t pooled_heads, int32_t* __restrict__ status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SelectHist* hist = reinterpret_cast<SelectHist*>(smem_raw);                // [8]
  float* qbar = reinterpret_cast<float*>(hist + 8);
  float* srows = qbar + (FROM_SCORES ? 0 : RMAX * D);                       // [RMAX][nb]

  const int64_t slot = blockIdx.y;
  const int64_t r0 = (int64_t)blockIdx.x * RMAX;
  const int rows = (int)(qb_count - r0 < RMAX ? qb_count - r0 : RMAX);
  const int tid = threadIdx.x;

  if constexpr (FROM_SCORES) {
    // rows are [slot*qb_count + r] of a [rows, nb] matrix
    for (int r = 0; r < rows; ++r) {
      const float* src = scores_in + (slot * qb_count + r0 + r) * nb;
      for (int64_t i = tid; i < nb; i += blockDim.x) srows[r * nb + i] = src[i];
    }
  } else {
    // pooled rows of this slot's head (with head_map: means of every head,
    // the slot picking its head)
    int64_t src = slot;
    if (head_map != nullptr) {
      src = head_map[slot];
      if (src < 0 || src >= pooled_heads) {
        if (tid == 0 && status) atomicOr(status, VGGT_STATUS_BAD_HEAD);
        for (int r = 0; r < rows; ++r) {
          const int64_t row = slot * qb_count + r0 + r;
          for (int64_t j = tid; j < max_blocks; j += blockDim.x) indices[row * max_blocks + j] = -1;
          if (tid == 0) counts[row] = 0;
        }
        return;
      }
    }
    const float* qsrc = pooled_q + (src * qb_count + r0) * D;
    for (int i = tid; i < rows * D; i += blockDim.x) qbar[i] = qsrc[i];
    for (int i = rows * D + tid; i < RMAX * D; i += blockDim.x) qbar[i] = 0.f;
    __syncthreads();
    const float* ksrc = pooled_k + src * nb * D;
    for (int64_t kb = tid; kb < nb; kb += blockDim.x) {
      // every row's dot product accumulates d = 0 .. D-1 in order (one fmaf
      // each); pooled K is streamed in 16-float chunks to keep registers low
      float acc[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) acc[r] = 0.f;
      const float4* kp = reinterpret_cast<const float4*>(ksrc + kb * D);
#pragma unroll
      for (int i0 = 0; i0 < D; i0 += 16) {
        float kv[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 t = __ldg(kp + i0 / 4 + i);
          kv[4 * i] = t.x; kv[4 * i + 1] = t.y; kv[4 * i + 2] = t.z; kv[4 * i + 3] = t.w;
        }
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          const float4* q4 = reinterpret_cast<const float4*>(qbar + r * D + i0);
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const float4 qv = q4[j4];  // warp-uniform: one broadcast 16-byte read
            acc[r] = fmaf(qv.x, kv[4 * j4], acc[r]);
            acc[r] = fmaf(qv.y, kv[4 * j4 + 1], acc[r]);
            acc[r] = fmaf(qv.z, kv[4 * j4 + 2], acc[r]);
            acc[r] = fmaf(qv.w, kv[4 * j4 + 3], acc[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < rows) {
          const float sc = acc[r] * scale;
          srows[r * nb + kb] = sc;
          if (scores_out) scores_out[(slot * qb_count + r0 + r) * nb + kb] = sc;
        }
      }
    }
  }
  __syncthreads();
  const int warp = tid >> 5;
  for (int r = warp; r < rows; r += (blockDim.x >> 5)) {
    const int64_t row = slot * qb_count + r0 + r;
    int m = select_row_warp(srows + (int64_t)r * nb, (int)nb, mode, topk, tau_num, hist + warp,
                            indices + row * max_blocks, max_blocks);
    if ((threadIdx.x & 31) == 0) counts[row] = m;
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
// Shared memory of one selection CTA holding `rows` score rows.
static size_t select_smem_bytes(int rows, int64_t nb, int d, bool from_scores) {
  return 8 * sizeof(SelectHist) + (size_t)rows * ((from_scores ? 0 : d) + nb) * 4;
}
constexpr size_t kSelectSmemBudget = 220 * 1024;

template <int D, bool FROM, int RMAX>
static cudaError_t launch_select_r(const float* pq, const float* pk, int64_t qb_count, int64_t nb,
                                   int64_t n_slots, float scale, int mode, int64_t topk,
                                   uint64_t tau_num, int32_t* indices, int64_t max_blocks,
                                   int32_t* counts, float* scores_out, const float* scores_in,
                                   const int32_t* head_map, int64_t pooled_heads, int32_t* status,
                                   cudaStream_t stream) {
  const size_t smem = select_smem_bytes(RMAX, nb, D, FROM);
  auto kern = score_select_kernel<D, FROM, RMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((qb_count + RMAX - 1) / RMAX), (unsigned)n_slots);
  kern<<<grid, 256, smem, stream>>>(pq, pk, qb_count, nb, scale, mode, topk, tau_num, indices,
                                     max_blocks, counts, scores_out, scores_in, head_map,
                                     pooled_heads, status);
  return cudaGetLastError();
}

// 8 query-block rows per CTA (one warp each) when they fit in shared memory,
// else 2 (very long rows).
template <int D, bool FROM>
static cudaError_t launch_select_t(const float* pq, const float* pk, int64_t qb_count, int64_t nb,
                                   int64_t n_slots, float scale, int mode, int64_t topk,
                                   uint64_t tau_num, int32_t* indices, int64_t max_blocks,
                                   int32_t* counts, float* scores_out, const float* scores_in,
                                   cudaStream_t stream, const int32_t* head_map = nullptr,
                                   int64_t pooled_heads = 0, int32_t* status = nullptr) {
  if (select_smem_bytes(8, nb, D, FROM) <= kSelectSmemBudget)
    return launch_select_r<D, FROM, 8>(pq, pk, qb_count, nb, n_slots, scale, mode, topk, tau_num,
                                       indices, max_blocks, counts, scores_out, scores_in,
                                       head_map, pooled_heads, status, stream);
  if (select_smem_bytes(2, nb, D, FROM) <= kSelectSmemBudget)
    return launch_select_r<D, FROM, 2>(pq, pk, qb_count, nb, n_slots, scale, mode, topk, tau_num,
                                       indices, max_blocks, counts, scores_out, scores_in,
                                       head_map, pooled_heads, status, stream);
  return cudaErrorInvalidValue;
}

int estimator_max_blocks_supported(int d) {
  // largest nb that still fits two rows per CTA
  return (int)((kSelectSmemBudget - 8 * sizeof(SelectHist)) / (2 * 4) - d);
}

template <typename T>
static cudaError_t launch_pool_t(const void* x, int64_t len, int d, int block, int64_t nblocks,
                                 const int32_t* head_ids, int64_t n_slots, int64_t heads,
                                 float* pooled, int32_t* status, cudaStream_t stream) {
  const int64_t units = n_slots * nblocks;
  const int warps = 8;
  dim3 grid((unsigned)((units + warps - 1) / warps));
  if (d == 64)
    pool_blocks_kernel<T, 64><<<grid, warps * 32, 0, stream>>>(
        static_cast<const T*>(x), len, block, nblocks, head_ids, n_slots, heads, pooled, status);
  else
    pool_blocks_kernel<T, 32><<<grid, warps * 32, 0, stream>>>(
        static_cast<const T*>(x), len, block, nblocks, head_ids, n_slots, heads, pooled, status);
  return cudaGetLastError();
}

cudaError_t launch_pool(const void* x, int dtype, int64_t len, int d, int block, int64_t nblocks,
                        const int32_t* head_ids, int64_t n_slots, int64_t heads, float* pooled,
                        int32_t* status, cudaStream_t stream) {
  if (units_zero(n_slots, nblocks)) return cudaSuccess;
  if (dtype == VGGT_DTYPE_BF16)
    return launch_pool_t<__nv_bfloat16>(x, len, d, block, nblocks, head_ids, n_slots, heads,
                                        pooled, status, stream);
  return launch_pool_t<__half>(x, len, d, block, nblocks, head_ids, n_slots, heads, pooled,
                               status, stream);
}

cudaError_t launch_score_select(const float* pq, const float* pk, int d, int64_t qb_count,
                                int64_t nb, int64_t n_slots, float scale, int mode, int64_t topk,
                                uint64_t tau_num, int32_t* indices, int64_t max_blocks,
                                int32_t* counts, float* scores_out, cudaStream_t stream) {
  if (units_zero(n_slots, qb_count)) return cudaSuccess;
  if (d == 64)
    return launch_select_t<64, false>(pq, pk, qb_count, nb, n_slots, scale, mode, topk, tau_num,
                                      indices, max_blocks, counts, scores_out, nullptr, stream);
  return launch_select_t<32, false>(pq, pk, qb_count, nb, n_slots, scale, mode, topk, tau_num,
                                    indices, max_blocks, counts, scores_out, nullptr, stream);
}

cudaError_t launch_score_select_mapped(const float* pq, const float* pk, int d, int64_t qb_count,
                                       int64_t nb, const int32_t* head_map, int64_t pooled_heads,
                                       int64_t n_slots, float scale, int mode, int64_t topk,
                                       uint64_t tau_num, int32_t* indices, int64_t max_blocks,
                                       int32_t* counts, float* scores_out, int32_t* status,
                                       cudaStream_t stream) {
  if (units_zero(n_slots, qb_count)) return cudaSuccess;
  if (d == 64)
    return launch_select_t<64, false>(pq, pk, qb_count, nb, n_slots, scale, mode, topk, tau_num,
                                      indices, max_blocks, counts, scores_out, nullptr, stream,
                                      head_map, pooled_heads, status);
  return launch_select_t<32, false>(pq, pk, qb_count, nb, n_slots, scale, mode, topk, tau_num,
                                    indices, max_blocks, counts, scores_out, nullptr, stream,
                                    head_map, pooled_heads, status);
}

cudaError_t launch_select_from_scores(const float* scores, int64_t rows, int64_t nb, int mode,
                                      int64_t topk, uint64_t tau_num, int32_t* indices,
                                      int64_t max_blocks, int32_t* counts, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  return launch_select_t<32, true>(nullptr, nullptr, rows, nb, 1, 1.f, mode, topk, tau_num,
                                   indices, max_blocks, counts, nullptr, scores, stream);
}

}  // namespace vggt
