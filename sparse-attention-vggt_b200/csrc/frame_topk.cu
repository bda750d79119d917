// Per-frame QK top-k on the 5th-generation tensor cores.
//
// Computes what saf3r/triton/fused_qk_topk.py:24-108 (_fused_perframe_qk_topk_kernel)
// and its launcher compute_qk_topk_indices_fused (:128-217) compute: for each
// query row and each frame of `tokens` consecutive keys, the indices of the
// frame's `topk` largest scores q . k (bf16 inputs, fp32 accumulation, no
// scale), in descending order, ties to the lower key index.  Scores are
// ordered by their sortable 32-bit keys (fpval_to_key, topk_utils.py:24-28):
// the float order, with +0 above -0.
//
// One CTA = 128 query rows of one batch entry x a contiguous group of frames.
//  * warp 0 (one lane): TMA.  The Q tile once, then 128-key K tiles, frame
//    aligned (tile j of frame f starts at key f * tokens + 128 j; keys past
//    the frame's end are masked, keys past the tensor's end read as zero),
//    into a ring of shared-memory stages.
//  * warp 1 (one lane): S = Q K^T with tcgen05 (both operands in shared
//    memory, fp32 accumulator in TMEM, two 128-column S buffers).
//  * warps 2-5: selection, one query row per thread (TMEM lane = row).  A
//    score passes if it is not below the row's current k-th best; passing
//    scores are appended to a per-row candidate buffer with predicated
//    shared-memory stores (no branch per score), then merged into the row's
//    list with every score checked exactly.  topk <= 8: a sorted list in
//    registers, seeded with the frame's first four scores; scores are
//    screened four at a time (a quad whose largest score passes is stored
//    whole) and merged every 64 columns.  Above 8: a min-heap in shared
//    memory; scores are screened one at a time and merged every 32 columns
//    (with a large top-k most quads would pass).  After a frame's last tile
//    the list is written out (in descending order) and reset.
//
// Every mbarrier wait is bounded (1 s); on expiry the CTA raises its abort
// flag, records VGGT_STATUS_TIMEOUT, drains its in-flight copies, frees its
// TMEM and exits.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace vggt {

namespace qktopk {

constexpr int BM = 128;                     // query rows per CTA
constexpr int BN = 128;                     // keys per tile
constexpr int THREADS = 192;
constexpr int CHUNK = 64;                   // columns between merges (half a tile)
constexpr int QUADS = CHUNK / 4;            // candidate slots: one 4-score quad each
constexpr int MAX_STAGES = 4;
constexpr uint32_t SPAN_BYTES = 128 * 128;  // 128 rows x 64 bf16: one 128-B swizzle span wide
constexpr uint32_t CAND_STRIDE = BM * 16;   // one slot of every row: 16 bytes per row
constexpr uint32_t CAND_BYTES = QUADS * CAND_STRIDE;
constexpr uint32_t TMEM_COLS = 256;         // two S buffers of 128 columns
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;

// barrier indices
constexpr int B_QFULL = 0;
constexpr int B_KFULL = 1;                        // [MAX_STAGES]
constexpr int B_KEMPTY = B_KFULL + MAX_STAGES;    // [MAX_STAGES]
constexpr int B_SFULL = B_KEMPTY + MAX_STAGES;    // [2]
constexpr int B_SEMPTY = B_SFULL + 2;             // [2]
constexpr int B_DRAIN = B_SEMPTY + 2;
constexpr int NBAR = B_DRAIN + 1;

struct Params {
  int32_t* out;      // [batch, n_queries, frames * topk]
  int32_t* status;
  int64_t n_queries, tokens, frames, qtiles, groups;
  int topk;          // entries per frame (<= tokens)
  int kch;           // 64-column spans of the head dim (1 or 2)
  int nstage;
  // shared-memory offsets from the 1024-aligned base
  uint32_t off_k, off_cand, off_list, off_bar;
};

struct Layout {
  uint32_t off_k, off_cand, off_list, off_bar, total;
  int nstage;
};

// Stages as many as fit (at most 4), the rest fixed.
inline Layout layout(int kch, int topk, bool list_in_smem) {
  Layout l;
  const uint32_t q_bytes = (uint32_t)kch * SPAN_BYTES;
  const uint32_t stage_bytes = (uint32_t)kch * SPAN_BYTES;
  const uint32_t list_bytes = list_in_smem ? (uint32_t)topk * BM * 8 : 0u;
  const uint32_t fixed = q_bytes + CAND_BYTES + list_bytes + NBAR * 8 + 64;
  const uint32_t budget = 227u * 1024u - 1024u;  // dynamic smem less the alignment slack
  int ns = fixed < budget ? (int)((budget - fixed) / stage_bytes) : 0;
  ns = ns > MAX_STAGES ? MAX_STAGES : ns;
  // two CTAs per SM when the ring of 3 fits in half the SM's shared memory
  if (ns >= 3 && fixed + 3 * stage_bytes + 1024 <= 112u * 1024u) ns = 3;
  l.nstage = ns;
  l.off_k = q_bytes;
  l.off_cand = l.off_k + (uint32_t)ns * stage_bytes;
  l.off_list = l.off_cand + CAND_BYTES;
  l.off_bar = l.off_list + list_bytes;
  l.total = l.off_bar + NBAR * 8 + 64 + 1024;
  // at most two CTAs per SM: the pair uses all 512 TMEM columns
  if (l.total < 80u * 1024u) l.total = 80u * 1024u;
  return l;
}

__device__ __forceinline__ uint32_t f2key(uint32_t bits) {
  return bits ^ ((uint32_t)((int32_t)bits >> 31) | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t key) {
  return __uint_as_float(key ^ (~(uint32_t)((int32_t)key >> 31) | 0x80000000u));
}

// Screens one quad of scores (columns 4Q .. 4Q+3 of a half tile): when the
// largest is not below `thr` (or any of the five is NaN) the four score bits
// are appended at `addr` (one 16-byte candidate slot), `addr` advances by one
// slot and bit Q of `mask` is set.  No branch.
template <int Q>
__device__ __forceinline__ void screen_quad(uint32_t& addr, uint32_t& mask, const uint32_t (&s)[64],
                                            float thr) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .f32 m;\n\t"
      "max.NaN.f32 m, %2, %3, %4;\n\t"
      "max.NaN.f32 m, m, %5;\n\t"
      "setp.geu.f32 p, m, %6;\n\t"
      "@p st.shared.v4.u32 [%0], {%7, %8, %9, %10};\n\t"
      "@p add.u32 %0, %0, %12;\n\t"
      "@p or.b32 %1, %1, %11;\n\t}"
      : "+r"(addr), "+r"(mask)
      : "f"(__uint_as_float(s[4 * Q])), "f"(__uint_as_float(s[4 * Q + 1])),
        "f"(__uint_as_float(s[4 * Q + 2])), "f"(__uint_as_float(s[4 * Q + 3])), "f"(thr),
        "r"(s[4 * Q]), "r"(s[4 * Q + 1]), "r"(s[4 * Q + 2]), "r"(s[4 * Q + 3]), "n"(1u << Q),
        "n"(CAND_STRIDE)
      : "memory");
}

// Quads Q .. QUADS-1 of a half tile; quads at or past column `lim` of the
// half are skipped (lim >= 64: none).
template <int Q>
__device__ __forceinline__ void screen_quads(uint32_t& addr, uint32_t& mask, const uint32_t (&s)[64],
                                             float thr, int lim) {
  if constexpr (Q < QUADS) {
    if (lim >= 64 || 4 * Q < lim) screen_quad<Q>(addr, mask, s, thr);
    screen_quads<Q + 1>(addr, mask, s, thr, lim);
  }
}

// The heap path screens score by score: with a large top-k most quads would
// pass.  Appends (score bits, column) as one 8-byte slot when the score is
// not below `thr` (or either is NaN) and advances `addr` by one slot.
__device__ __forceinline__ void screen_one(uint32_t& addr, uint32_t bits, float thr, uint32_t col) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.geu.f32 p, %1, %2;\n\t"
      "@p st.shared.v2.u32 [%0], {%3, %4};\n\t"
      "@p add.u32 %0, %0, %5;\n\t}"
      : "+r"(addr)
      : "f"(__uint_as_float(bits)), "f"(thr), "r"(bits), "r"(col), "n"(BM * 8)
      : "memory");
}

__device__ __forceinline__ uint2 ld_shared_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// The row's sorted list: keys descending, an equal key after the earlier
// (lower-index) entry.  Key 0 marks an empty slot (no float maps to 0 except
// the NaN with every bit set, which is never inserted).
template <int KR>
struct RegList {  // topk <= KR <= 8: registers
  uint32_t key[KR], idx[KR];
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int i = 0; i < KR; ++i) key[i] = 0u;
  }
  __device__ __forceinline__ uint32_t last() const { return key[KR - 1]; }
  // requires k > last()
  __device__ __forceinline__ void insert(uint32_t k, uint32_t ix) {
#pragma unroll
    for (int i = KR - 1; i > 0; --i) {
      const bool shift = key[i - 1] < k;  // the new entry ranks above entry i - 1
      const bool here = !shift && key[i] < k;
      const uint32_t nk = shift ? key[i - 1] : (here ? k : key[i]);
      const uint32_t ni = shift ? idx[i - 1] : (here ? ix : idx[i]);
      key[i] = nk;
      idx[i] = ni;
    }
    if (key[0] < k) {
      key[0] = k;
      idx[0] = ix;
    }
  }
  __device__ __forceinline__ void write(int32_t* dst, int topk, int32_t base) const {
    if (KR == 4 && topk == 4) {
      int4 v;
      v.x = key[0] ? base + (int32_t)idx[0] : -1;
      v.y = key[1] ? base + (int32_t)idx[1] : -1;
      v.z = key[2] ? base + (int32_t)idx[2] : -1;
      v.w = key[3] ? base + (int32_t)idx[3] : -1;
      *reinterpret_cast<int4*>(dst) = v;
      return;
    }
#pragma unroll
    for (int i = 0; i < KR; ++i)
      if (i < topk) dst[i] = key[i] ? base + (int32_t)idx[i] : -1;
  }
};

// topk <= 128: a min-heap in shared memory ([slot][row], so a warp's rows are
// contiguous) of 64-bit composites (key << 32 | ~index): the root is the
// row's current k-th best.  An insert replaces the root and sifts it down;
// the frame's list is heap-sorted into descending order when written out.
// Slots start at composite 0, below every real entry.
struct HeapList {
  unsigned long long* h;
  int k, row;
  uint32_t root_key;
  __device__ __forceinline__ void reset() {
    for (int i = 0; i < k; ++i) h[i * BM + row] = 0ull;
    root_key = 0u;
  }
  __device__ __forceinline__ uint32_t last() const { return root_key; }
  __device__ __forceinline__ void sift(unsigned long long c, int i, int n) {
    while (true) {
      const int l = 2 * i + 1;
      if (l >= n) break;
      unsigned long long cc = h[l * BM + row];
      int child = l;
      if (l + 1 < n) {
        const unsigned long long cr = h[(l + 1) * BM + row];
        if (cr < cc) {
          cc = cr;
          child = l + 1;
        }
      }
      if (cc >= c) break;
      h[i * BM + row] = cc;
      i = child;
    }
    h[i * BM + row] = c;
  }
  // requires kn > last(): the new entry beats the root
  __device__ __forceinline__ void insert(uint32_t kn, uint32_t ix) {
    sift(((unsigned long long)kn << 32) | (unsigned long long)(0xffffffffu - ix), 0, k);
    root_key = (uint32_t)(h[row] >> 32);
  }
  // heap-sorts in place (descending from slot 0) and writes the first topk
  __device__ __forceinline__ void write(int32_t* dst, int topk, int32_t base) {
    for (int n = k - 1; n > 0; --n) {
      const unsigned long long top = h[row];
      const unsigned long long tail = h[n * BM + row];
      h[n * BM + row] = top;
      sift(tail, 0, n);
    }
    for (int i = 0; i < topk; ++i) {
      const unsigned long long c = h[i * BM + row];
      dst[i] = c ? base + (int32_t)(0xffffffffu - (uint32_t)c) : -1;
    }
  }
};

template <int KR>
__global__ void __launch_bounds__(THREADS, 2)
    frame_topk_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k, Params p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw_addr);
  const uint32_t bar0 = base + p.off_bar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(sbase + p.off_bar + NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ns = p.nstage;

  // ---- work decode: consecutive CTAs take the frame groups of one Q tile ----
  const int64_t g = blockIdx.x % p.groups;
  const int64_t rest = blockIdx.x / p.groups;
  const int64_t qt = rest % p.qtiles;
  const int64_t b = rest / p.qtiles;
  const int64_t f0 = p.frames * g / p.groups;
  const int64_t f1 = p.frames * (g + 1) / p.groups;
  const int tpf = (int)((p.tokens + BN - 1) / BN);  // tiles per frame
  const int64_t n_tiles = (f1 - f0) * tpf;

  if (tid == 0) {
    tc::mbar_init(bar(B_QFULL), 1);
    for (int s = 0; s < ns; ++s) {
      tc::mbar_init(bar(B_KFULL + s), 1);
      tc::mbar_init(bar(B_KEMPTY + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(bar(B_SFULL + s), 1);
      tc::mbar_init(bar(B_SEMPTY + s), 128);
    }
    tc::mbar_init(bar(B_DRAIN), 1);
    misc[1] = 0u;
    tc::mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(base + p.off_bar + NBAR * 8, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = misc[0];
  auto t_s = [tmem](int buf) { return tmem + (uint32_t)(buf * BN); };
  const uint32_t span = SPAN_BYTES;
  const uint32_t stage_bytes = (uint32_t)p.kch * span;

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      tc::prefetch_tmap(&tm_q);
      tc::prefetch_tmap(&tm_k);
      tc::mbar_expect_tx(bar(B_QFULL), stage_bytes);
      for (int c = 0; c < p.kch; ++c)
        tc::tma_load_3d(base + (uint32_t)c * span, &tm_q, bar(B_QFULL), c * 64, (int)(qt * BM),
                        (int)b);
      int64_t issued = 0;
      for (int64_t t = 0; t < n_tiles; ++t) {
        const int stage = (int)(t % ns);
        if (t >= ns && !tc::mbar_wait(bar(B_KEMPTY + stage), (uint32_t)((t / ns - 1) & 1),
                                      abort_flag, WAIT_LIMIT_NS))
          break;
        const int64_t f = f0 + t / tpf;
        const int64_t row = f * p.tokens + (t % tpf) * BN;
        tc::mbar_expect_tx(bar(B_KFULL + stage), stage_bytes);
        for (int c = 0; c < p.kch; ++c)
          tc::tma_load_3d(base + p.off_k + (uint32_t)stage * stage_bytes + (uint32_t)c * span,
                          &tm_k, bar(B_KFULL + stage), c * 64, (int)row, (int)b);
        ++issued;
      }
      if (*abort_flag) {
        tc::mbar_wait_drain(bar(B_QFULL), 0, WAIT_LIMIT_NS);
        const int64_t first = issued > ns ? issued - ns : 0;
        for (int64_t t = first; t < issued; ++t)
          tc::mbar_wait_drain(bar(B_KFULL + (int)(t % ns)), (uint32_t)((t / ns) & 1),
                              WAIT_LIMIT_NS);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(1u, 0u, BM, BN);  // bf16, K-major A and B
      bool ok = tc::mbar_wait(bar(B_QFULL), 0, abort_flag, WAIT_LIMIT_NS);
      for (int64_t t = 0; ok && t < n_tiles; ++t) {
        const int stage = (int)(t % ns);
        const int buf = (int)(t & 1);
        if (!tc::mbar_wait(bar(B_KFULL + stage), (uint32_t)((t / ns) & 1), abort_flag,
                           WAIT_LIMIT_NS) ||
            (t >= 2 && !tc::mbar_wait(bar(B_SEMPTY + buf), (uint32_t)(((t >> 1) - 1) & 1),
                                      abort_flag, WAIT_LIMIT_NS))) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        for (int c = 0; c < p.kch; ++c) {
          const uint64_t qd = tc::sw128_desc(base + (uint32_t)c * span, 16);
          const uint64_t kd =
              tc::sw128_desc(base + p.off_k + (uint32_t)stage * stage_bytes + (uint32_t)c * span, 16);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_ss(t_s(buf), qd + (uint64_t)(kk * 2), kd + (uint64_t)(kk * 2), idesc,
                       (c > 0 || kk > 0) ? 1u : 0u);
        }
        tc::mma_commit(bar(B_KEMPTY + stage));
        tc::mma_commit(bar(B_SFULL + buf));
      }
      tc::mma_commit(bar(B_DRAIN));
      tc::mbar_wait_drain(bar(B_DRAIN), 0, WAIT_LIMIT_NS);
    }
  } else {
    // ================= selection: warps 2..5, one query row per thread ============
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const int64_t qrow = qt * BM + row;
    const bool valid_row = qrow < p.n_queries;
    const uint32_t cand_row = base + p.off_cand + (uint32_t)row * 16u;
    typename std::conditional<(KR > 0), RegList<(KR > 0 ? KR : 1)>, HeapList>::type list;
    if constexpr (KR == 0) {
      list.h = reinterpret_cast<unsigned long long*>(sbase + p.off_list);
      list.k = p.topk;
      list.row = row;
    }
    int32_t* out_row =
        p.out + ((b * p.n_queries + (valid_row ? qrow : 0)) * p.frames) * (int64_t)p.topk;
    float thr = __uint_as_float(0xffffffffu);  // NaN: every score passes
    bool ok = true;

    // Inserts the half tile's passing quads in column order (an equal key
    // then lands after the earlier, lower-index entry); every score of a
    // quad is checked exactly against the list, columns >= lim skipped.
    auto merge = [&](uint32_t addr, uint32_t mask, uint32_t col0, int lim) {
      const int cnt = (int)((addr - cand_row) / CAND_STRIDE);
      const int mc = __reduce_max_sync(0xffffffffu, cnt);
      for (int c = 0; c < mc; ++c) {
        if (c < cnt) {
          const int qd = __ffs(mask) - 1;
          mask &= mask - 1u;
          const uint4 e = ld_shared_v4(cand_row + (uint32_t)c * CAND_STRIDE);
          const uint32_t v[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int col = 4 * qd + i;
            const uint32_t key = f2key(v[i]);
            if (col < lim && key > list.last()) list.insert(key, col0 + (uint32_t)col);
          }
        }
      }
      thr = key2f(list.last());
    };

    for (int64_t t = 0; t < n_tiles; ++t) {
      const int buf = (int)(t & 1);
      const int j = (int)(t % tpf);
      const int64_t f = f0 + t / tpf;
      if (j == 0) {
        list.reset();
        thr = __uint_as_float(0xffffffffu);
      }
      const bool got =
          tc::mbar_wait(bar(B_SFULL + buf), (uint32_t)((t >> 1) & 1), abort_flag, WAIT_LIMIT_NS);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      const int64_t rem = p.tokens - (int64_t)j * BN;
      const int vc = rem < BN ? (int)rem : BN;  // valid columns of this tile
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t s[64];
        __syncwarp();
        tc::tmem_ld32(t_s(buf) + lane_off + (uint32_t)(h * 64), s);
        tc::tmem_ld32(t_s(buf) + lane_off + (uint32_t)(h * 64 + 32), s + 32);
        tc::tmem_wait_ld();
        if (h == 1) {
          tc::tc_fence_before();
          tc::mbar_arrive(bar(B_SEMPTY + buf));
        }
        const int lim = vc - h * 64;  // valid columns of this half
        if (lim <= 0) continue;       // uniform: the half is past the frame
        const uint32_t col0 = (uint32_t)(j * BN + h * 64);
        if constexpr (KR == 0) {
          // heap: 32-column chunks of 8-byte (score, column) slots
          const uint32_t row8 = base + p.off_cand + (uint32_t)row * 8u;
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            if (c2 * 32 >= lim) break;  // uniform
            uint32_t addr = row8;
            if (c2 * 32 + 32 <= lim) {
#pragma unroll
              for (int i = 0; i < 32; ++i) screen_one(addr, s[c2 * 32 + i], thr, col0 + c2 * 32 + i);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (c2 * 32 + i < lim) screen_one(addr, s[c2 * 32 + i], thr, col0 + c2 * 32 + i);
            }
            const int cnt = (int)((addr - row8) / (BM * 8));
            const int mc = __reduce_max_sync(0xffffffffu, cnt);
            for (int c = 0; c < mc; ++c) {
              if (c < cnt) {
                const uint2 e = ld_shared_v2(row8 + (uint32_t)c * (BM * 8));
                const uint32_t key = f2key(e.x);
                if (key > list.last()) list.insert(key, e.y);
              }
            }
            thr = key2f(list.last());
          }
          continue;
        }
        uint32_t addr = cand_row, mask = 0u;
        {
          if (j == 0 && h == 0) {
            // the frame's first quad goes straight into the empty list, so
            // the screen starts with a real k-th best
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t key = f2key(s[i]);
              if (i < lim && key > list.last()) list.insert(key, (uint32_t)i);
            }
            thr = key2f(list.last());
            screen_quads<1>(addr, mask, s, thr, lim);
          } else {
            screen_quads<0>(addr, mask, s, thr, lim);
          }
        }
        merge(addr, mask, col0, lim);
      }
      if (j == tpf - 1 && valid_row)
        list.write(out_row + f * p.topk, p.topk, (int32_t)(f * p.tokens));
    }
    (void)ok;
  }

  tc::tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag && p.status) atomicOr(p.status, VGGT_STATUS_TIMEOUT);
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int KR>
cudaError_t launch_t(const CUtensorMap& mq, const CUtensorMap& mk, const Params& p,
                     uint32_t smem, int64_t grid, cudaStream_t stream) {
  auto k = frame_topk_kernel<KR>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<(unsigned)grid, THREADS, smem, stream>>>(mq, mk, p);
  return cudaGetLastError();
}

}  // namespace qktopk

bool frame_topk_supported(int dim, int64_t topk) {
  return (dim == 64 || dim == 128) && topk >= 1 && topk <= 128;
}

int64_t frame_topk_groups(int64_t frames, int64_t work_rows) {
  // about 8 waves of 2 CTAs per SM, a group holding at least one frame
  constexpr int64_t kTarget = 8 * 2 * 148;
  if (frames <= 1 || work_rows <= 0) return 1;
  int64_t g = (kTarget + work_rows - 1) / work_rows;
  return g > frames ? frames : (g < 1 ? 1 : g);
}

cudaError_t launch_frame_topk(const FrameTopkArgs& a, cudaStream_t stream) {
  using namespace qktopk;
  if (a.batch == 0 || a.n_queries == 0 || a.frames == 0) return cudaSuccess;
  CUtensorMap mq, mk;
  if (!encode_tmap_3d_sw128(&mq, a.q, VGGT_DTYPE_BF16, a.dim, a.n_queries, a.batch, 64, BM) ||
      !encode_tmap_3d_sw128(&mk, a.k, VGGT_DTYPE_BF16, a.dim, a.frames * a.tokens, a.batch, 64,
                            BN))
    return cudaErrorInvalidValue;
  const int kr = a.topk <= 4 ? 4 : (a.topk <= 8 ? 8 : 0);
  Params p;
  p.out = a.out;
  p.status = a.status;
  p.n_queries = a.n_queries;
  p.tokens = a.tokens;
  p.frames = a.frames;
  p.qtiles = (a.n_queries + BM - 1) / BM;
  p.topk = (int)a.topk;
  p.kch = a.dim / 64;
  const Layout l = layout(p.kch, p.topk, kr == 0);
  if (l.nstage < 1) return cudaErrorInvalidValue;
  p.nstage = l.nstage;
  p.off_k = l.off_k;
  p.off_cand = l.off_cand;
  p.off_list = l.off_list;
  p.off_bar = l.off_bar;
  p.groups = a.groups > 0 ? a.groups : frame_topk_groups(a.frames, p.qtiles * a.batch);
  if (p.groups > a.frames) p.groups = a.frames;
  const int64_t grid = p.qtiles * a.batch * p.groups;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  switch (kr) {
    case 4:
      return launch_t<4>(mq, mk, p, l.total, grid, stream);
    case 8:
      return launch_t<8>(mq, mk, p, l.total, grid, stream);
    default:
      return launch_t<0>(mq, mk, p, l.total, grid, stream);
  }
}

}  // namespace vggt
