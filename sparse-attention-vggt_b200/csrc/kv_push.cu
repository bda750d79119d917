// Frame-shard exchange of K/V over NVLink peer memory.
//
// In the sequence-parallel layer every rank holds the patch and special K/V
// of its own frames ([heads, n_local, d] per tensor) and needs every frame's.
// Each rank's buffers live in one symmetric allocation (the same size and
// layout on every rank, each rank's mapped into every other's address
// space).  This kernel stores the rank's shard rows of every head straight
// into every rank's head-major full buffers ([heads, world * n_local, d],
// rows [rank * n_local, (rank + 1) * n_local)), so no staging buffer, no
// reordering copy and no library collective sits between the shards and the
// attention kernel.  Stores only: nothing here reads another GPU's memory,
// and there is no TMA and no multicast.
//
// Ordering, with a flag area of uint32 words at the end of each rank's
// allocation and an epoch that the host raises by one per exchange:
//  * handshake (the first phase of an exchange): the launch is ordered after
//    this rank's previous readers of its full buffers; the first CTA to
//    start tells every rank so (ready[rank] = epoch in each rank's flags),
//    and every CTA then waits until all ranks have said the same before it
//    stores into their buffers;
//  * after its stores every CTA fences at system scope and counts itself
//    done; the last one signals every rank (done[phase][rank] = epoch, a
//    release store) and then waits until every rank has signalled it, so
//    the launch completes only once this rank's full buffers hold every
//    rank's rows.
// Every wait is bounded (wait_ns); on expiry the launch ORs
// VGGT_STATUS_TIMEOUT into *status, and the buffers are then invalid.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace vggt {

namespace kvpush {

// flag words per rank allocation
__device__ __forceinline__ int ready_word(int j) { return j; }
__device__ __forceinline__ int done_word(int world, int phase, int j) {
  return world + phase * world + j;
}
__device__ __forceinline__ int start_cnt_word(int world, int phase) { return 3 * world + phase; }
__device__ __forceinline__ int end_cnt_word(int world, int phase) { return 3 * world + 2 + phase; }

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// waits (bounded) until flag word `w` of this rank's area is at least epoch
// for every rank; false on expiry
__device__ bool wait_all(const uint32_t* flags, int first_word, int world, uint32_t epoch,
                         uint64_t limit_ns) {
  const uint64_t t0 = tc::globaltimer_ns();
  for (int j = 0; j < world; ++j) {
    while ((int32_t)(ld_acquire_sys(flags + first_word + j) - epoch) < 0) {
      if (tc::globaltimer_ns() - t0 > limit_ns) return false;
      __nanosleep(128);
    }
  }
  return true;
}

__global__ void __launch_bounds__(256) kv_push_kernel(KvPushArgs a) {
  uint32_t* flags = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(a.peers[a.rank]) +
                                                a.flags_off);
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    bool ok = true;
    if (a.handshake) {
      if (atomicAdd(flags + start_cnt_word(a.world, a.phase), 1u) == 0u) {
        for (int j = 0; j < a.world; ++j)
          st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(a.peers[j]) +
                                                     a.flags_off) + ready_word(a.rank),
                         a.epoch);
      }
      ok = wait_all(flags, ready_word(0), a.world, a.epoch, a.wait_ns);
    }
    s_ok = ok;
    if (!ok && a.status) atomicOr(a.status, VGGT_STATUS_TIMEOUT);
  }
  __syncthreads();
  if (s_ok) {
    const int64_t total = a.unit_end[a.n_tensors - 1];
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += stride) {
      int t = 0;
      while (t + 1 < a.n_tensors && u >= a.unit_end[t]) ++t;
      const int64_t lu = u - (t ? a.unit_end[t - 1] : 0);   // unit within tensor t's shard
      const int64_t row = lu / a.row_units;                 // head * n_local + local row
      const int64_t part = lu - row * a.row_units;
      const int64_t h = row / a.rows_local[t];
      const int64_t r = row - h * a.rows_local[t];
      const uint4 v = __ldg(a.src[t] + lu);
      const int64_t dst = (h * a.rows_local[t] * a.world + (int64_t)a.rank * a.rows_local[t] + r) *
                              a.row_units + part;
      for (int j = 0; j < a.world; ++j)
        reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.peers[j]) + a.dst_off[t])[dst] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's stores before its count
    uint32_t* ecnt = flags + end_cnt_word(a.world, a.phase);
    if (atomicAdd(ecnt, 1u) == gridDim.x - 1) {
      // the last CTA: every CTA's stores are ordered before its count
      __threadfence_system();
      *ecnt = 0u;
      if (a.handshake) flags[start_cnt_word(a.world, a.phase)] = 0u;
      for (int j = 0; j < a.world; ++j)
        st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(a.peers[j]) +
                                                   a.flags_off) +
                           done_word(a.world, a.phase, a.rank),
                       a.epoch);
      if (!wait_all(flags, done_word(a.world, a.phase, 0), a.world, a.epoch, a.wait_ns) &&
          a.status)
        atomicOr(a.status, VGGT_STATUS_TIMEOUT);
      __threadfence_system();
    }
  }
}

}  // namespace kvpush

cudaError_t launch_kv_push(const KvPushArgs& a, int grid, cudaStream_t stream) {
  kvpush::kv_push_kernel<<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace vggt
