// Query-block pairing for the tcgen05 attention kernel.
//
// The tcgen05 kernel runs two 64-row query blocks per 128-row tile over the
// union of their key-block selections (a tile selected by only one of them is
// masked for the other's rows), so a pair costs |A u B| tiles for |A| + |B|
// tile-rows of useful work.  Pairing each query block with a block whose
// selection differs least (Hamming distance of the two selection bitmaps,
// |A xor B| = 2|A u B| - |A| - |B|) cuts that waste: on clustered multi-view
// inputs adjacent blocks waste 10-25% of the sparse tile work, the pairs
// chosen here 2-4%.  The pairing changes only which rows share a tile; every
// row still sees exactly its own key set in ascending block order, so the
// attention output is bit-identical to the adjacent pairing.
//
// Four launches on the caller's stream (the pairs are deterministic):
//   1. bitmap: one warp per (slot, query block) turns the index list into a
//      selection bitmap (built in shared memory, stored coalesced).
//   2. cost:   cost[slot][a][d-1] = popcount(bm[a] ^ bm[a + d]) for the
//      PAIR_WINDOW blocks after a, tiled through shared memory word chunk by
//      word chunk.
//   3. greedy: one warp per slot walks the query blocks in order; an unpaired
//      block a takes the unpaired candidate a + d (d <= PAIR_WINDOW) of least
//      cost (ties -> smallest d); blocks left without a candidate are paired
//      with each other in order at the end.  Cost rows stream through a
//      double-buffered shared-memory window; the taken flags of the
//      candidate window stay in registers.  Each pair's union size is kept.
//   4. schedule: the attention grid's work order: slots in the natural order,
//      each slot's pairs by descending size (the grid ends on short CTAs).
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace vggt {

namespace pairing {

constexpr int W = PAIR_WINDOW;       // candidates after each block
constexpr int BM_WARPS = 8;          // bitmap kernel: warps per CTA
constexpr int COST_ROWS = 32;        // cost kernel: a-blocks per CTA
constexpr int COST_CHUNK = 16;       // cost kernel: bitmap words per smem chunk
constexpr int COST_THREADS = 256;
constexpr int GREEDY_ROWS = 32;      // greedy kernel: cost rows per smem buffer

__global__ void __launch_bounds__(BM_WARPS * 32)
    bitmap_kernel(const int32_t* __restrict__ indices, const int32_t* __restrict__ counts,
                  int counts_per_qblock, const uint8_t* __restrict__ head_dense, int64_t n_slots, int64_t qb_count, int64_t max_blocks,
                  int64_t nb, int nwords, uint32_t* __restrict__ bitmaps) {
  extern __shared__ uint32_t sbm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* mine = sbm + (size_t)warp * nwords;
  const int64_t row = (int64_t)blockIdx.x * BM_WARPS + warp;  // slot * qb_count + qb
  if (row >= n_slots * qb_count) return;
  const int64_t slot = row / qb_count;
  if (head_dense != nullptr && head_dense[slot]) return;  // no index rows
  for (int i = lane; i < nwords; i += 32) mine[i] = 0u;
  __syncwarp();
  int64_t cnt = counts_per_qblock ? counts[row] : counts[slot];
  cnt = cnt < 0 ? 0 : (cnt > max_blocks ? max_blocks : cnt);
  const int32_t* ids = indices + row * max_blocks;
  for (int64_t i = lane; i < cnt; i += 32) {
    const int32_t kb = ids[i];
    if (kb >= 0 && kb < nb) atomicOr(&mine[kb >> 5], 1u << (kb & 31));
  }
  __syncwarp();
  uint32_t* dst = bitmaps + row * nwords;
  for (int i = lane; i < nwords; i += 32) dst[i] = mine[i];
}

// grid (ceil(qb_count / COST_ROWS), n_slots).  Each thread owns
// COST_ROWS * W / COST_THREADS (a, d) pairs and accumulates their popcounts
// over the bitmap words, COST_CHUNK words at a time from shared memory.
__global__ void __launch_bounds__(COST_THREADS)
    cost_kernel(const uint32_t* __restrict__ bitmaps, const uint8_t* __restrict__ head_dense,
                int64_t qb_count, int nwords, uint16_t* __restrict__ cost) {
  constexpr int SPAN = COST_ROWS + W;  // bitmaps a CTA needs
  constexpr int PER = COST_ROWS * W / COST_THREADS;
  __shared__ uint32_t chunk[SPAN][COST_CHUNK + 1];
  const int64_t slot = blockIdx.y;
  if (head_dense != nullptr && head_dense[slot]) return;
  const int64_t a0 = (int64_t)blockIdx.x * COST_ROWS;
  const uint32_t* bm = bitmaps + slot * qb_count * (int64_t)nwords;
  uint32_t acc[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) acc[k] = 0u;
  for (int w0 = 0; w0 < nwords; w0 += COST_CHUNK) {
    __syncthreads();
    for (int i = threadIdx.x; i < SPAN * COST_CHUNK; i += COST_THREADS) {
      const int r = i / COST_CHUNK, w = i % COST_CHUNK;
      const int64_t blk = a0 + r;
      chunk[r][w] = (blk < qb_count && w0 + w < nwords) ? bm[blk * nwords + w0 + w] : 0u;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int pidx = threadIdx.x + k * COST_THREADS;
      const int r = pidx / W, d = pidx % W + 1;
      uint32_t s = 0u;
#pragma unroll
      for (int w = 0; w < COST_CHUNK; ++w) s += __popc(chunk[r][w] ^ chunk[r + d][w]);
      acc[k] += s;
    }
  }
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int pidx = threadIdx.x + k * COST_THREADS;
    const int r = pidx / W, d = pidx % W + 1;
    const int64_t a = a0 + r;
    if (a < qb_count)
      cost[(slot * qb_count + a) * W + (d - 1)] =
          (a + d < qb_count) ? (uint16_t)(acc[k] > 0xfffeu ? 0xfffeu : acc[k]) : (uint16_t)0xffffu;
  }
}

// One warp per slot.  pairs [n_slots, ceil(qb_count / 2), 2]; singles is
// scratch [n_slots, qb_count].  Which of the candidates a + 1 .. a + W are
// already taken lives in registers: lane L holds the bits of d = 4L+1 .. 4L+4,
// and the window slides by one block per step with one shuffle (a block
// beyond a + W can only have been taken by a block after a, so zeros shift
// in).
__global__ void __launch_bounds__(32)
    greedy_kernel(const uint16_t* __restrict__ cost, const uint8_t* __restrict__ head_dense,
                  const int32_t* __restrict__ counts, int counts_per_qblock, int64_t max_blocks,
                  int64_t qb_count, int32_t* __restrict__ pairs, int32_t* __restrict__ sizes,
                  int32_t* __restrict__ singles) {
  extern __shared__ unsigned char gsm[];
  uint16_t* rows = reinterpret_cast<uint16_t*>(gsm);  // [2][GREEDY_ROWS][W]
  const int lane = threadIdx.x;
  const unsigned full = 0xffffffffu;
  const int64_t slot = blockIdx.x;
  if (head_dense != nullptr && head_dense[slot]) return;  // the kernel pairs dense slots itself
  const uint16_t* crow = cost + slot * qb_count * W;
  int32_t* out = pairs + slot * ((qb_count + 1) / 2) * 2;
  int32_t* osize = sizes + slot * ((qb_count + 1) / 2);
  int32_t* single = singles + slot * qb_count;
  // selected blocks of query block q (clamped as the attention kernel clamps)
  auto count_of = [&](int64_t q) -> int32_t {
    int64_t c = counts_per_qblock ? counts[slot * qb_count + q] : counts[slot];
    return (int32_t)(c < 0 ? 0 : (c > max_blocks ? max_blocks : c));
  };
  static_assert(W == 128, "4 candidates per lane");
  // the next GREEDY_ROWS cost rows are fetched into registers while the
  // current ones are walked, then stored to the other buffer
  constexpr int NF = GREEDY_ROWS * W / 8 / 32;  // uint4 per lane per buffer
  uint4 pre[NF];
  auto fetch = [&](int64_t r0) {
#pragma unroll
    for (int j = 0; j < NF; ++j) {
      const int i = lane + 32 * j;
      const int64_t r = r0 + (i * 8) / W;
      pre[j] = r < qb_count ? *reinterpret_cast<const uint4*>(crow + r0 * W + (int64_t)i * 8)
                            : make_uint4(0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu);
    }
  };
  auto store = [&](int buf) {
    uint16_t* dst = rows + (size_t)buf * GREEDY_ROWS * W;
#pragma unroll
    for (int j = 0; j < NF; ++j) *reinterpret_cast<uint4*>(dst + (lane + 32 * j) * 8) = pre[j];
  };
  fetch(0);
  store(0);
  __syncwarp();
  uint32_t tk = 0u;        // taken bits of this lane's 4 candidates
  bool cur_taken = false;  // block a itself
  int64_t np = 0, ns = 0;
  for (int64_t base = 0; base < qb_count; base += GREEDY_ROWS) {
    const int buf = (int)((base / GREEDY_ROWS) & 1);
    const bool more = base + GREEDY_ROWS < qb_count;
    if (more) fetch(base + GREEDY_ROWS);
    const uint16_t* cur = rows + (size_t)buf * GREEDY_ROWS * W;
    const int64_t lim = more ? base + GREEDY_ROWS : qb_count;
    for (int64_t a = base; a < lim; ++a) {
      if (!cur_taken) {
        // this lane's 4 costs: d = 4 lane + 1 .. 4 lane + 4
        const uint2 c4 = *reinterpret_cast<const uint2*>(cur + (a - base) * W + 4 * lane);
        const uint32_t cs[4] = {c4.x & 0xffffu, c4.x >> 16, c4.y & 0xffffu, c4.y >> 16};
        uint32_t best = 0xffffffffu;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int d = 4 * lane + k + 1;
          if (a + d < qb_count && cs[k] != 0xffffu && !((tk >> k) & 1u)) {
            const uint32_t key = (cs[k] << 16) | (uint32_t)d;
            best = key < best ? key : best;
          }
        }
        best = __reduce_min_sync(full, best);
        if (best != 0xffffffffu) {
          const int d = (int)(best & 0xffffu);
          if (lane == ((d - 1) >> 2)) tk |= 1u << ((d - 1) & 3);
          if (lane == 0) {
            out[2 * np] = (int32_t)a;
            out[2 * np + 1] = (int32_t)(a + d);
            // tiles of the union: (|A| + |B| + |A xor B|) / 2
            osize[np] = (count_of(a) + count_of(a + d) + (int32_t)(best >> 16)) / 2;
          }
          ++np;
        } else {
          if (lane == 0) single[ns] = (int32_t)a;
          ++ns;
        }
      }
      // slide the window to a + 1: block a + 1 (d = 1, lane 0 bit 0) becomes
      // the current block; lane L's bits take d + 1 from itself and lane L + 1
      cur_taken = (__shfl_sync(full, tk, 0) & 1u) != 0u;
      const uint32_t up = __shfl_down_sync(full, tk, 1);
      tk = (tk >> 1) | ((lane < 31 ? (up & 1u) : 0u) << 3);
    }
    __syncwarp();
    if (more) store(buf ^ 1);
    __syncwarp();
  }
  // leftover blocks pair with each other in order (the last one alone if odd)
  __syncwarp();
  for (int64_t i = lane; 2 * i < ns; i += 32) {
    const int32_t x = single[2 * i];
    const int32_t y = 2 * i + 1 < ns ? single[2 * i + 1] : -1;
    out[2 * (np + i)] = x;
    out[2 * (np + i) + 1] = y;
    osize[np + i] = count_of(x) + (y >= 0 ? count_of(y) : 0);  // an upper bound
  }
}

// One CTA per slot: the slots keep the natural launch order (the last slot,
// where the dense-profiled heads sit, first), so the CTAs in flight share one
// or two heads' K/V in L2; within a slot the pairs go by descending tile
// count, so the grid ends on the shortest items.  Sizes fall into
// SCHED_BUCKETS equal-width buckets of [0, nb]; the order within a bucket is
// whatever the atomics give (it only changes which CTA runs when).
constexpr int SCHED_BUCKETS = 1024;
__global__ void __launch_bounds__(256)
    schedule_kernel(const int32_t* __restrict__ sizes, const uint8_t* __restrict__ head_dense,
                    int64_t n_slots, int64_t npairs, int64_t nb, int32_t* __restrict__ order) {
  __shared__ int hist[SCHED_BUCKETS];
  const int64_t slot = blockIdx.x;
  int32_t* dst = order + (n_slots - 1 - slot) * npairs;
  if (head_dense != nullptr && head_dense[slot]) {  // every pair walks all nb blocks
    for (int64_t i = threadIdx.x; i < npairs; i += blockDim.x) dst[i] = (int32_t)(slot * npairs + i);
    return;
  }
  for (int i = threadIdx.x; i < SCHED_BUCKETS; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int32_t* sz = sizes + slot * npairs;
  auto bucket_of = [&](int64_t i) -> int {
    int64_t v = sz[i];
    v = v < 0 ? 0 : (v > nb ? nb : v);
    return (int)((v * (SCHED_BUCKETS - 1)) / (nb > 0 ? nb : 1));
  };
  for (int64_t i = threadIdx.x; i < npairs; i += blockDim.x) atomicAdd(&hist[bucket_of(i)], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    // exclusive offsets from the largest bucket down
    int run = 0;
    for (int b = SCHED_BUCKETS - 1; b >= 0; --b) {
      const int c = hist[b];
      hist[b] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < npairs; i += blockDim.x)
    dst[atomicAdd(&hist[bucket_of(i)], 1)] = (int32_t)(slot * npairs + i);
}

}  // namespace pairing

size_t qblock_pairing_workspace(int64_t n_slots, int64_t qb_count, int64_t nb) {
  const int64_t nwords = (nb + 31) / 32;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  return up((size_t)n_slots * qb_count * nwords * 4) +        // bitmaps
         up((size_t)n_slots * qb_count * PAIR_WINDOW * 2) +   // costs
         up((size_t)n_slots * qb_count * 4) +                 // singles
         up((size_t)n_slots * ((qb_count + 1) / 2) * 4);      // pair sizes
}

bool qblock_pairing_supported(int64_t qb_count, int64_t nb) {
  // bitmap kernel: 8 warps' bitmaps of nb bits in shared memory
  return qb_count >= 2 && qb_count <= 0x7fffffffLL && nb >= 1 && nb <= 65536;
}

cudaError_t launch_qblock_pairing(const int32_t* indices, const int32_t* counts,
                                  int counts_per_qblock, const uint8_t* head_dense, int64_t n_slots,
                                  int64_t qb_count, int64_t max_blocks, int64_t nb, int32_t* pairs,
                                  int32_t* order, void* workspace, cudaStream_t stream) {
  using namespace pairing;
  if (n_slots == 0) return cudaSuccess;
  const int nwords = (int)((nb + 31) / 32);
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  uint32_t* bitmaps = reinterpret_cast<uint32_t*>(ws);
  ws += up((size_t)n_slots * qb_count * nwords * 4);
  uint16_t* cost = reinterpret_cast<uint16_t*>(ws);
  ws += up((size_t)n_slots * qb_count * W * 2);
  int32_t* singles = reinterpret_cast<int32_t*>(ws);
  ws += up((size_t)n_slots * qb_count * 4);
  int32_t* sizes = reinterpret_cast<int32_t*>(ws);

  const int64_t rows = n_slots * qb_count;
  const size_t smem_bm = (size_t)BM_WARPS * nwords * 4;
  cudaError_t e = cudaFuncSetAttribute(bitmap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_bm);
  if (e != cudaSuccess) return e;
  bitmap_kernel<<<(unsigned)((rows + BM_WARPS - 1) / BM_WARPS), BM_WARPS * 32, smem_bm, stream>>>(
      indices, counts, counts_per_qblock, head_dense, n_slots, qb_count, max_blocks, nb, nwords,
      bitmaps);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cost_kernel<<<dim3((unsigned)((qb_count + COST_ROWS - 1) / COST_ROWS), (unsigned)n_slots),
                COST_THREADS, 0, stream>>>(bitmaps, head_dense, qb_count, nwords, cost);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem_g = 2 * GREEDY_ROWS * W * sizeof(uint16_t);
  e = cudaFuncSetAttribute(greedy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem_g);
  if (e != cudaSuccess) return e;
  greedy_kernel<<<(unsigned)n_slots, 32, smem_g, stream>>>(
      cost, head_dense, counts, counts_per_qblock, max_blocks, qb_count, pairs, sizes, singles);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  schedule_kernel<<<(unsigned)n_slots, 256, 0, stream>>>(sizes, head_dense, n_slots,
                                                        (qb_count + 1) / 2, nb, order);
  return cudaGetLastError();
}

}  // namespace vggt
