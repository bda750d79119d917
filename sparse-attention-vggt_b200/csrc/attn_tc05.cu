// Block-sparse attention forward on the 5th-generation tensor cores.
//
// Computes what saf3r/triton/adaptive_block_attention.py:7-60 computes (exact
// softmax over each query block's selected 64-key patch blocks plus all
// special keys, fp32 online softmax) with a different decomposition:
//
//  * one CTA = 128 query rows = two adjacent 64-row query blocks (2p, 2p+1)
//    of one slot (head).  The key tiles are the ascending union of the two
//    blocks' selections; a tile selected by only one block is masked to -inf
//    for the other block's 64 rows, so every output row sees exactly its own
//    key set.  This keeps tcgen05 at M=128, its full-rate shape.
//  * each softmax thread loads its query row once into TMEM (the A operand of
//    QK^T, 32 columns).  Warp 0 (one lane) streams K and V tiles with TMA
//    (3-D tensor maps over [heads, rows, 64], 128-byte swizzle, zero fill past
//    the end of a head) into a 4-stage ring; warp 1 (one lane) issues
//      S_t  = Q K_t^T  (TS: Q from TMEM, K from smem; fp32 S double-buffered)
//      O   += P_t V_t  (TS: P read from TMEM where it overwrote S_t; O stays
//                       in TMEM for the whole key sweep)
//    and warps 2-5 (128 threads, one query row each) run the softmax: read
//    S_t, mask tail columns, exp2(s * scale * log2 e - m_ref) with one FFMA
//    per element, write P_t (bf16/fp16) back to TMEM in two column halves,
//    each with its own full barrier, so the MMA lane issues the first half's
//    PV MMAs while the second half's exponentials run.  A softmax warp probes
//    its tile's K/V-full and S-full barriers back to back (both are usually
//    complete) and only then falls back to the bounded waits.  The per-row reference
//    max m_ref only moves when a tile's max exceeds it by more than 8 in the
//    exp2 domain; O (in TMEM) and the row sum are rescaled then, so P <= 2^8
//    and the rescale is rare after the first tiles.
//  * dense-profiled slots walk every patch block (no index reads): the dense
//    path of the same kernel.
//
// Every mbarrier wait is bounded (Params.wait_ns, 1 s by default; the drains
// below always allow 1 s); on expiry the CTA raises an abort
// flag, records VGGT_STATUS_TIMEOUT, drains its in-flight copies, frees its
// TMEM and exits.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"



namespace vggt {

namespace tcattn {

constexpr int BM = 128;         // query rows per CTA
constexpr int BN = 64;          // keys per tile
constexpr int HD = 64;          // head dim
#ifndef VGGT_TC_NSTAGE
#define VGGT_TC_NSTAGE 4
#endif
constexpr int NSTAGE = VGGT_TC_NSTAGE;  // K/V ring depth
#ifndef VGGT_TC_PAIRED_PROBE
#define VGGT_TC_PAIRED_PROBE 1
#endif
constexpr int THREADS = 192;
constexpr uint32_t TILE_BYTES = BN * HD * 2;  // 8 KB
constexpr uint32_t TMEM_COLS = 256;  // S0 | S1 | O (64 + 16 row-sum cols) | Q: 2 CTAs/SM
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;

// shared-memory layout (offsets from a 1024-aligned base)
constexpr uint32_t OFF_K = 0;
constexpr uint32_t OFF_V = OFF_K + NSTAGE * TILE_BYTES;
// A 64x64 tile of ones, read as N columns 64..79 of the PV MMA's B operand:
// O[:, 64] then accumulates the row sum of P on the tensor core.
constexpr uint32_t OFF_ONES = OFF_V + NSTAGE * TILE_BYTES;
constexpr uint32_t OFF_BAR = OFF_ONES + TILE_BYTES;
constexpr int ON = 80;  // PV MMA N: 64 value columns + 16 ones columns
// barrier indices
constexpr int B_QFULL = 0;
constexpr int B_KVFULL = 1;                 // [NSTAGE]
constexpr int B_KVEMPTY = B_KVFULL + NSTAGE;  // [NSTAGE]
constexpr int B_SFULL = B_KVEMPTY + NSTAGE;   // [2]
// P is published in P_PARTS column parts of 64 / P_PARTS keys each
#ifndef VGGT_TC_P_PARTS
#define VGGT_TC_P_PARTS 2
#endif
constexpr int P_PARTS = VGGT_TC_P_PARTS;
static_assert(P_PARTS == 2 || P_PARTS == 4, "P parts: 2 or 4");
constexpr int PAIRS_PER_PART = 32 / P_PARTS;  // packed P columns per part
constexpr int B_PFULL = B_SFULL + 2;          // [2 buffers][P_PARTS]
constexpr int B_PVDONE = B_PFULL + 2 * P_PARTS;  // one phase per PV MMA
constexpr int B_OFULL = B_PVDONE + 1;         // the last PV MMA is done
constexpr int B_DRAIN = B_OFULL + 1;          // MMA completion before TMEM release
constexpr int B_NEVER = B_DRAIN + 1;          // nothing arrives (wait self-test)
constexpr int NBAR = B_NEVER + 1;
constexpr uint32_t OFF_META = OFF_BAR + NBAR * 8;       // int[NSTAGE]
constexpr uint32_t OFF_MISC = OFF_META + NSTAGE * 4;    // tmem base, abort, tiles, scratch
// evidence partials: float[4 ring][2 query blocks][2 warps] + int counters[4][2]
constexpr uint32_t OFF_EV = (OFF_MISC + 64 + 15) & ~15u;
constexpr uint32_t OFF_BITMAP = OFF_EV + 4 * 2 * 2 * 4 + 4 * 2 * 4;
// (bitmaps, then for evidence the uint16 slot index of each block per query block)

struct Params {
  const void* q;
  const int32_t* indices;
  const int32_t* counts;
  const int32_t* head_ids;
  const uint8_t* head_dense;
  void* out;
  int32_t* status;
  int64_t heads, n_tokens, n_patch, n_special, n_slots, max_blocks, qb_count, nb, pairs;
  float* evidence;  // [n_slots, qb_count, max_blocks] or null
  const int32_t* pair_table;  // [indexed slots, pairs, 2] or null
  const int32_t* work_order;  // [n_slots * pairs] work items in launch order, or null
  // Split of each work item's tile list over nsplit CTAs (1 = none).  With
  // nsplit > 1 a CTA writes its unnormalised O, row sum and reference max to
  // `partial` ([item][split][66][128] fp32) and split 0 the destination row of
  // each of its 128 rows to `part_rows` ([item][128], -1 = none); the combine
  // kernel then writes `out`.
  int nsplit;
  float* partial;
  int64_t* part_rows;
  int counts_per_qblock;
  float scale_log2;
  uint64_t wait_ns;  // limit of every pipeline wait (the drains keep WAIT_LIMIT_NS)
  // failure-detection self-test: the MMA issuer first waits on B_NEVER, which
  // runs out after wait_ns and aborts the CTA through the normal path
  int wait_selftest;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA/ALU pipes, for x <= 8 (the lazy-rescale bound).  Range
// reduction x = n + f with n = round(x) (adding 1.5 * 2^23 leaves round(x) in
// the low mantissa bits), f in [-1/2, 1/2]; 2^f by a cubic fitted to minimise
// the maximum relative error on that interval (iteratively reweighted least
// squares, max relative error 7.5e-5, below bf16/fp16 resolution); the result
// exponent is then advanced by n with one integer add.  x is clamped at -126
// so the exponent field stays valid (2^-126 is negligible next to P <= 2^8).
#ifndef VGGT_TC_POLY_PAIRS
#define VGGT_TC_POLY_PAIRS 0x01u
#endif
#ifndef VGGT_TC_EXP_F16X2
#define VGGT_TC_EXP_F16X2 0
#endif
// column pairs (of every 8) whose exponentials run on the FMA pipe
constexpr unsigned kPolyPairs = VGGT_TC_POLY_PAIRS;

// (d0, d1) = (a0, a1) * b + c with one packed f32x2 FMA
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %4};\n\t"
      "mov.b64 rc, {%5, %5};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}

__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = __fadd_rn(x, 12582912.f);
  const float n = __fsub_rn(t, 12582912.f);
  const float f = __fsub_rn(x, n);
  float q = fmaf(f, 0.05517131f, 0.24261053f);
  q = fmaf(q, f, 0.69326099f);
  q = fmaf(q, f, 0.99992811f);
  return __int_as_float(__float_as_int(q) + (__float_as_int(t) << 23));
}

#ifndef VGGT_TC_POLY_F32X2
#define VGGT_TC_POLY_F32X2 1
#endif

// two polynomial exponentials, packed into the MMA element type.  With
// VGGT_TC_POLY_F32X2 the pair shares one chain of packed f32x2 instructions
// (same steps, same cubic, same result bits as exp2_poly on each element):
// the rounding add and the two subtractions are explicit .rn operations, so
// nothing contracts them into an FMA and the round-to-integer trick holds.
template <typename T>
__device__ __forceinline__ uint32_t exp2_poly_pair(float xa, float xb) {
#if VGGT_TC_POLY_F32X2
  xa = fmaxf(xa, -126.f);
  xb = fmaxf(xb, -126.f);
  float qa, qb, ta, tb;
  asm("{\n\t.reg .b64 x, m, t, n, f, q, c3, c2, c1, c0;\n\t"
      "mov.b64 x, {%4, %5};\n\t"
      "mov.b64 m, {%6, %6};\n\t"
      "mov.b64 c3, {%7, %7};\n\t"
      "mov.b64 c2, {%8, %8};\n\t"
      "mov.b64 c1, {%9, %9};\n\t"
      "mov.b64 c0, {%10, %10};\n\t"
      "add.rn.f32x2 t, x, m;\n\t"
      "sub.rn.f32x2 n, t, m;\n\t"
      "sub.rn.f32x2 f, x, n;\n\t"
      "fma.rn.f32x2 q, f, c3, c2;\n\t"
      "fma.rn.f32x2 q, q, f, c1;\n\t"
      "fma.rn.f32x2 q, q, f, c0;\n\t"
      "mov.b64 {%0, %1}, q;\n\t"
      "mov.b64 {%2, %3}, t;\n\t}"
      : "=f"(qa), "=f"(qb), "=f"(ta), "=f"(tb)
      : "f"(xa), "f"(xb), "f"(12582912.f), "f"(0.05517131f), "f"(0.24261053f),
        "f"(0.69326099f), "f"(0.99992811f));
  return ElemOps<T>::pack2(__int_as_float(__float_as_int(qa) + (__float_as_int(ta) << 23)),
                           __int_as_float(__float_as_int(qb) + (__float_as_int(tb) << 23)));
#else
  return ElemOps<T>::pack2(exp2_poly(xa), exp2_poly(xb));
#endif
}

// two MUFU exponentials, packed into the MMA element type.  With
// VGGT_TC_EXP_F16X2 the pair is rounded to f16 (11-bit significand; for the
// x <= 8 range here the argument error is <= 2^-8) and one ex2.f16x2 computes
// both; otherwise two fp32 ex2.
template <typename T>
__device__ __forceinline__ uint32_t exp2_mufu_pair(float xa, float xb) {
#if VGGT_TC_EXP_F16X2
  uint32_t h, e;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(xb), "f"(xa));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(h));
  if constexpr (std::is_same<T, __half>::value) {
    return e;
  } else {
    const float2 f = __half22float2(*reinterpret_cast<__half2*>(&e));
    return ElemOps<T>::pack2(f.x, f.y);
  }
#else
  return ElemOps<T>::pack2(ex2(xa), ex2(xb));
#endif
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <typename T, bool EVID>
__global__ void __launch_bounds__(THREADS, 2)
    attn_tc05_kernel(const __grid_constant__ CUtensorMap tm_kp,
                     const __grid_constant__ CUtensorMap tm_vp,
                     const __grid_constant__ CUtensorMap tm_ks,
                     const __grid_constant__ CUtensorMap tm_vs, Params p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw_addr);
  const uint32_t bar0 = base + OFF_BAR;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  volatile int* meta = reinterpret_cast<volatile int*>(sbase + OFF_META);
  uint32_t* misc = reinterpret_cast<uint32_t*>(sbase + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  uint32_t* bm = reinterpret_cast<uint32_t*>(sbase + OFF_BITMAP);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- work decode: the given order, else dense-heavy slots (last in the
  // slot order) first; consecutive CTAs take the splits of one item ----
  const int64_t w = blockIdx.x / p.nsplit;
  const int split = (int)(blockIdx.x % p.nsplit);
  int64_t slot = p.n_slots - 1 - w / p.pairs;
  int64_t pair = w % p.pairs;
  if (p.work_order != nullptr) {
    const int64_t item = p.work_order[w];
    if (item < 0 || item >= p.n_slots * p.pairs) {
      if (tid == 0 && p.status) atomicOr(p.status, VGGT_STATUS_BAD_INDEX);
      return;
    }
    slot = item / p.pairs;
    pair = item % p.pairs;
  }
  const int64_t head = p.head_ids[slot];
  if (head < 0 || head >= p.heads) {
    if (tid == 0 && p.status) atomicOr(p.status, VGGT_STATUS_BAD_HEAD);
    return;
  }
  const bool dense = p.head_dense != nullptr && p.head_dense[slot] != 0;
  // the tile's two query blocks: (2p, 2p + 1), or an entry of the pair table
  int64_t qb0 = 2 * pair, qb1 = qb0 + 1;
  if (!dense && p.pair_table != nullptr) {
    qb0 = p.pair_table[2 * (slot * p.pairs + pair)];
    qb1 = p.pair_table[2 * (slot * p.pairs + pair) + 1];
    if (qb0 < 0 || qb0 >= p.qb_count || qb1 < -1 || qb1 >= p.qb_count || qb1 == qb0) {
      if (tid == 0 && p.status) atomicOr(p.status, VGGT_STATUS_BAD_INDEX);
      return;
    }
  }
  const bool has1 = qb1 >= 0 && qb1 < p.qb_count;
  const int nwords = (int)((p.nb + 31) >> 5);
  uint32_t* bmA = bm;
  uint32_t* bmB = bm + nwords;
  // slot of each selected block in its query block's index list (evidence only)
  uint16_t* invA = reinterpret_cast<uint16_t*>(bm + 2 * nwords);
  uint16_t* invB = invA + ((p.nb + 7) & ~7LL);
  float* ev_part = reinterpret_cast<float*>(sbase + OFF_EV);
  int* ev_cnt = reinterpret_cast<int*>(ev_part + 16);

  // ---- union of the two query blocks' selections as two bitmaps ----
  int64_t n_patch_tiles;
  if (dense) {
    n_patch_tiles = p.nb;
  } else {
    int64_t c0 = p.counts_per_qblock ? p.counts[slot * p.qb_count + qb0] : p.counts[slot];
    int64_t c1 = has1 ? (p.counts_per_qblock ? p.counts[slot * p.qb_count + qb1] : c0) : 0;
    if (c0 < 0 || c0 > p.max_blocks || c1 < 0 || c1 > p.max_blocks) {
      if (tid == 0 && p.status) atomicOr(p.status, VGGT_STATUS_BAD_COUNT);
      c0 = c0 < 0 ? 0 : (c0 > p.max_blocks ? p.max_blocks : c0);
      c1 = c1 < 0 ? 0 : (c1 > p.max_blocks ? p.max_blocks : c1);
    }
    for (int i = tid; i < 2 * nwords; i += THREADS) bm[i] = 0u;
    if (tid == 0) misc[2] = 0u;
    __syncthreads();
    const int32_t* row0 = p.indices + (slot * p.qb_count + qb0) * p.max_blocks;
    const int32_t* row1 = p.indices + (slot * p.qb_count + (has1 ? qb1 : qb0)) * p.max_blocks;
    bool bad = false;
    for (int64_t i = tid; i < c0; i += THREADS) {
      const int32_t kb = row0[i];
      if (kb >= 0 && kb < p.nb) {
        atomicOr(&bmA[kb >> 5], 1u << (kb & 31));
        if (EVID) invA[kb] = (uint16_t)i;
      } else {
        bad = true;
      }
    }
    for (int64_t i = tid; i < c1; i += THREADS) {
      const int32_t kb = row1[i];
      if (kb >= 0 && kb < p.nb) {
        atomicOr(&bmB[kb >> 5], 1u << (kb & 31));
        if (EVID) invB[kb] = (uint16_t)i;
      } else {
        bad = true;
      }
    }
    if (bad && p.status) atomicOr(p.status, VGGT_STATUS_BAD_INDEX);
    __syncthreads();
    uint32_t cnt = 0;
    for (int i = tid; i < nwords; i += THREADS) cnt += __popc(bmA[i] | bmB[i]);
    for (int off = 16; off; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
    if (lane == 0 && cnt) atomicAdd(&misc[2], cnt);
    __syncthreads();
    n_patch_tiles = misc[2];
  }
  const int64_t n_spec_tiles = (p.n_special + BN - 1) / BN;
  // this CTA's share [t0, t0 + n_tiles) of the item's tiles (patch tiles in
  // ascending order, then the special tiles)
  const int64_t n_all = n_patch_tiles + n_spec_tiles;
  const int64_t t0 = n_all * split / p.nsplit;
  const int64_t n_tiles = n_all * (split + 1) / p.nsplit - t0;

  // ---- barriers and TMEM ----
  if (tid == 0) {
    tc::mbar_init(bar(B_QFULL), 128);
    for (int s = 0; s < NSTAGE; ++s) {
      tc::mbar_init(bar(B_KVFULL + s), 1);
      tc::mbar_init(bar(B_KVEMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar(B_SFULL + b), 1);
      for (int hh = 0; hh < P_PARTS; ++hh) tc::mbar_init(bar(B_PFULL + P_PARTS * b + hh), 128);
    }
    tc::mbar_init(bar(B_PVDONE), 1);
    tc::mbar_init(bar(B_OFULL), 1);
    tc::mbar_init(bar(B_DRAIN), 1);
    tc::mbar_init(bar(B_NEVER), 1);
    misc[1] = 0u;  // abort flag
    for (int i = 0; i < 8; ++i) ev_cnt[i] = 0;
    tc::mbar_fence_init();
  }
  {
    // ones tile (1.0 in the element type); made visible to the tensor core below
    const uint32_t one2 = ElemOps<T>::pack2(1.f, 1.f);
    uint4* ones = reinterpret_cast<uint4*>(sbase + OFF_ONES);
    for (int i = tid; i < (int)(TILE_BYTES / 16); i += THREADS)
      ones[i] = make_uint4(one2, one2, one2, one2);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    tc::tmem_alloc(base + OFF_MISC, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = misc[0];
  // S buffer b lives at columns [64 b, 64 b + 64)
  auto t_s_of = [tmem](int b) { return tmem + (uint32_t)(b << 6); };
  const uint32_t t_o = tmem + 128u;
  const uint32_t t_q = tmem + 208u;  // Q tile as the A operand of QK (32 cols)

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      tc::prefetch_tmap(&tm_kp);
      tc::prefetch_tmap(&tm_vp);
      int wi = 0;
      uint32_t cur = 0, curA = 0;
      if (!dense && nwords > 0) {
        curA = bmA[0];
        cur = curA | bmB[0];
        // skip the union's first t0 blocks (earlier splits' tiles)
        int64_t skip = t0 < n_patch_tiles ? t0 : n_patch_tiles;
        while (skip > 0) {
          const int c = __popc(cur);
          if (c <= skip) {
            skip -= c;
            ++wi;
            if (wi < nwords) {
              curA = bmA[wi];
              cur = curA | bmB[wi];
            } else {
              cur = 0u;
            }
          } else {
            for (int64_t k = 0; k < skip; ++k) cur &= cur - 1u;
            skip = 0;
          }
        }
      }
      int64_t issued = 0;
      for (int64_t t = 0; t < n_tiles; ++t) {
        const int64_t g = t0 + t;  // index in the item's tile list
        const int stage = (int)(t % NSTAGE);
        if (t >= NSTAGE) {
          if (!tc::mbar_wait(bar(B_KVEMPTY + stage), (uint32_t)((t / NSTAGE - 1) & 1), abort_flag,
                             p.wait_ns))
            break;
        }
        int flags, ncols, row;
        const CUtensorMap *mk, *mv;
        if (g < n_patch_tiles) {
          int64_t kb;
          if (dense) {
            kb = g;
            flags = 3;
          } else {
            while (cur == 0u) {
              ++wi;
              curA = bmA[wi];
              cur = curA | bmB[wi];
            }
            const int b = __ffs(cur) - 1;
            cur &= cur - 1u;
            kb = (int64_t)wi * 32 + b;
            flags = (int)((curA >> b) & 1u) | (int)(((bmB[wi] >> b) & 1u) << 1);
          }
          row = (int)(kb * BN);
          ncols = (int)(p.n_patch - kb * BN < BN ? p.n_patch - kb * BN : BN);
          mk = &tm_kp;
          mv = &tm_vp;
        } else {
          const int64_t st = g - n_patch_tiles;
          flags = 3;
          row = (int)(st * BN);
          ncols = (int)(p.n_special - st * BN < BN ? p.n_special - st * BN : BN);
          mk = &tm_ks;
          mv = &tm_vs;
        }
        if (t == n_tiles - 1) flags |= 4;
        const bool special = g >= n_patch_tiles;
        // bits 0-1 query-block flags, 2 last, 3 special, 4-10 valid columns,
        // 12-31 patch block id
        meta[stage] = flags | (special ? 8 : 0) | (ncols << 4) |
                      ((special ? 0 : row / BN) << 12);
        tc::mbar_expect_tx(bar(B_KVFULL + stage), 2 * TILE_BYTES);
        tc::tma_load_3d(base + OFF_K + stage * TILE_BYTES, mk, bar(B_KVFULL + stage), 0, row,
                        (int)head);
        tc::tma_load_3d(base + OFF_V + stage * TILE_BYTES, mv, bar(B_KVFULL + stage), 0, row,
                        (int)head);
        ++issued;
      }
      {
        // drain: wait (bounded) for the last NSTAGE copies, landed or not, so
        // none is in flight when the CTA exits (after an abort the consumers
        // stop waiting for them; their completion depends on the copy alone)
        const int64_t first = issued > NSTAGE ? issued - NSTAGE : 0;
        for (int64_t t = first; t < issued; ++t)
          tc::mbar_wait_drain(bar(B_KVFULL + (int)(t % NSTAGE)), (uint32_t)((t / NSTAGE) & 1),
                              WAIT_LIMIT_NS);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t id_qk = tc::idesc_f16(fmt, 0u, BM, BN);
      const uint32_t id_pv = tc::idesc_f16(fmt, 1u, BM, ON);
      bool ok = tc::mbar_wait(bar(B_QFULL), 0, abort_flag, p.wait_ns);
      if (p.wait_selftest) ok = ok && tc::mbar_wait(bar(B_NEVER), 0, abort_flag, p.wait_ns);
      // O (TMEM) += P_u V_u; the first PV of the CTA initialises O.
      auto issue_pv = [&](int64_t u) -> bool {
        const int bu = (int)(u & 1);
        const int su = (int)(u % NSTAGE);
        // MN group 0 = the V tile, group 1 (LBO bytes further) = the ones tile
        const uint64_t vdesc = tc::sw128_desc(base + OFF_V + su * TILE_BYTES,
                                              OFF_ONES - (OFF_V + su * TILE_BYTES));
        // P arrives in P_PARTS column parts; each part's K = 16 MMAs go as
        // soon as it is published
        constexpr int MMAS = (BN / 16) / P_PARTS;
#pragma unroll
        for (int hh = 0; hh < P_PARTS; ++hh) {
          if (!tc::mbar_wait(bar(B_PFULL + P_PARTS * bu + hh), (uint32_t)((u >> 1) & 1),
                             abort_flag, p.wait_ns))
            return false;
          tc::tc_fence_after();
#pragma unroll
          for (int kk = MMAS * hh; kk < MMAS * hh + MMAS; ++kk)
            tc::mma_ts(t_o, t_s_of(bu) + (uint32_t)(kk * 8), vdesc + (uint64_t)(kk * 128), id_pv,
                       (u > 0 || kk > 0) ? 1u : 0u);
        }
        tc::mma_commit(bar(B_PVDONE));
        tc::mma_commit(bar(B_KVEMPTY + su));
        return true;
      };
      for (int64_t t = 0; ok && t < n_tiles; ++t) {
        const int stage = (int)(t % NSTAGE);
        const int b = (int)(t & 1);
        if (!tc::mbar_wait(bar(B_KVFULL + stage), (uint32_t)((t / NSTAGE) & 1), abort_flag,
                           p.wait_ns)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint64_t kdesc = tc::sw128_desc(base + OFF_K + stage * TILE_BYTES, 16);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          tc::mma_ts(t_s_of(b), t_q + (uint32_t)(kk * 8), kdesc + (uint64_t)(kk * 2), id_qk,
                     kk > 0 ? 1u : 0u);
        tc::mma_commit(bar(B_SFULL + b));
        if (t >= 1 && !issue_pv(t - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && n_tiles > 0 && issue_pv(n_tiles - 1)) tc::mma_commit(bar(B_OFULL));
      // every issued MMA must finish before the TMEM columns are released
      tc::mma_commit(bar(B_DRAIN));
      tc::mbar_wait_drain(bar(B_DRAIN), 0, WAIT_LIMIT_NS);
    }
  } else {
    // ================= softmax: warps 2..5, one query row per thread ============
    const int sub = warp & 3;                 // TMEM lane quarter of this warp
    const int row = sub * 32 + lane;          // 0..127
    const int half = row >> 6;                // which query block of the pair
    const int64_t my_qb = half ? (has1 ? qb1 : -1) : qb0;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const float c = p.scale_log2;
    {
      // this thread's query row -> TMEM (A operand layout: 2 elements per column)
      const int64_t qrow = my_qb * 64 + (row & 63);
      uint32_t r[32];
      if (my_qb >= 0 && qrow < p.n_tokens) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) +
                                                          (head * p.n_tokens + qrow) * HD);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint4 v = __ldg(src + k);
          r[4 * k] = v.x; r[4 * k + 1] = v.y; r[4 * k + 2] = v.z; r[4 * k + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) r[k] = 0u;
      }
      tc::tmem_st32(t_q + lane_off, r);
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(bar(B_QFULL));
    }
    // O accumulates in TMEM against a per-row reference max m_ref (raw score
    // units).  m_ref moves only when a tile's max exceeds it by more than
    // 2^8 in the exp2 domain; O (value and row-sum columns) is rescaled then
    // (P stays <= 256).
    float m_ref = -INFINITY;
    bool has_mass = false, ok = true;

    for (int64_t t = 0; t < n_tiles; ++t) {
      const int stage = (int)(t % NSTAGE);
      const int b = (int)(t & 1);
#if VGGT_TC_PAIRED_PROBE
      // both barriers are usually complete by now: probe them back to back so
      // the two probes' latencies overlap, and fall back to the bounded waits
      // only for one that is not
      const bool kv_ready = tc::mbar_try_wait(bar(B_KVFULL + stage), (uint32_t)((t / NSTAGE) & 1));
      const bool s_ready = tc::mbar_try_wait(bar(B_SFULL + b), (uint32_t)((t >> 1) & 1));
      bool got = (kv_ready || tc::mbar_wait(bar(B_KVFULL + stage), (uint32_t)((t / NSTAGE) & 1),
                                            abort_flag, p.wait_ns)) &&
                 (s_ready || tc::mbar_wait(bar(B_SFULL + b), (uint32_t)((t >> 1) & 1),
                                           abort_flag, p.wait_ns));
#else
      bool got = tc::mbar_wait(bar(B_KVFULL + stage), (uint32_t)((t / NSTAGE) & 1), abort_flag,
                               p.wait_ns) &&
                 tc::mbar_wait(bar(B_SFULL + b), (uint32_t)((t >> 1) & 1), abort_flag,
                               p.wait_ns);
#endif
      // keep the warp converged for the .sync.aligned TMEM instructions
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      const int mt = meta[stage];
      const int ncols = (mt >> 4) & 0x7f;
      const bool active = (mt >> half) & 1;
      tc::tc_fence_after();
      uint32_t s[64];
      tc::tmem_ld32(t_s_of(b) + lane_off, s);
      tc::tmem_ld32(t_s_of(b) + lane_off + 32u, s + 32);
      tc::tmem_wait_ld();
      uint32_t pk[32];
      // P is published in column parts (keys 0-31, then 32-63, with two
      // parts), so the MMA issuer starts a part's PV MMAs while the next
      // part's exponentials run.  `done` pairs of pk are complete.
      auto publish = [&](int hh, const uint32_t* src) {
        if constexpr (PAIRS_PER_PART == 16)
          tc::tmem_st16(t_s_of(b) + lane_off + (uint32_t)(PAIRS_PER_PART * hh), src);
        else
          tc::tmem_st8(t_s_of(b) + lane_off + (uint32_t)(PAIRS_PER_PART * hh), src);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        tc::mbar_arrive(bar(B_PFULL + P_PARTS * b + hh));
      };
      auto publish_done = [&](int done) {  // called after pair done - 1
        if (done % PAIRS_PER_PART == 0)
          publish(done / PAIRS_PER_PART - 1, pk + done - PAIRS_PER_PART);
      };
      if (active) {  // warp-uniform: a warp's 32 rows belong to one query block
        if (ncols < BN) {
#pragma unroll
          for (int i = 0; i < BN; ++i)
            if (i >= ncols) s[i] = __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mx[j] = fmax3(__uint_as_float(s[8 * j]),
                        fmax3(__uint_as_float(s[8 * j + 1]), __uint_as_float(s[8 * j + 2]),
                              __uint_as_float(s[8 * j + 3])),
                        fmax3(__uint_as_float(s[8 * j + 4]), __uint_as_float(s[8 * j + 5]),
                              fmaxf(__uint_as_float(s[8 * j + 6]), __uint_as_float(s[8 * j + 7]))));
        const float mloc = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]),
                                 fmaxf(mx[6], mx[7]));
        const bool grow = (mloc - m_ref) * c > 8.f;   // always true while m_ref = -inf
        const float m_new = grow ? mloc : m_ref;
        const float factor = grow ? ex2((m_ref - m_new) * c) : 1.f;  // 0 when m_ref = -inf
        const bool rescale_o = grow && has_mass;  // rows without mass have O == 0
        if (__any_sync(0xffffffffu, rescale_o)) {
          // O must hold every PV issued so far (through tile t-1) before it is
          // rescaled; PV_t cannot start before P_t is published below.
          const bool done = tc::mbar_wait(bar(B_PVDONE), (uint32_t)((t - 1) & 1), abort_flag,
                                          p.wait_ns);
          if (!__all_sync(0xffffffffu, done)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const float f = rescale_o ? factor : 1.f;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t r[32];
            tc::tmem_ld32(t_o + lane_off + 32u * h2, r);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
            tc::tmem_st32(t_o + lane_off + 32u * h2, r);
          }
          {  // the row-sum column
            uint32_t r[8];
            tc::tmem_ld8(t_o + lane_off + 64u, r);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
            tc::tmem_st8(t_o + lane_off + 64u, r);
          }
        }
        m_ref = m_new;
        has_mass = true;
        const float mc = m_ref * c;
        if constexpr (EVID) {
          // Same-pass evidence (adaptive_block_attention.py:29-33): the row's
          // log-sum-exp over this tile's keys, from the fp32 weights of the
          // same exponentials (all on MUFU here), averaged over the query
          // block's valid rows.  The two warps of a query block combine their
          // partial sums through shared memory; the second one stores.
          float sum = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float xa, xb;
            ffma2(xa, xb, __uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]), c, -mc);
            const float ea = ex2(xa), eb = ex2(xb);
            sum += ea + eb;
            pk[i] = ElemOps<T>::pack2(ea, eb);
            publish_done(i + 1);
          }
          if (!(mt & 8) && !dense) {  // patch tiles of indexed slots only
            const int64_t qrow = my_qb * 64 + (row & 63);
            float v = my_qb >= 0 && qrow < p.n_tokens ? (mc + __log2f(sum)) * 0.6931471805599453f : 0.f;
#pragma unroll
            for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) {
              const int slotr = (int)(t & 3) * 2 + half;
              ev_part[slotr * 2 + (sub & 1)] = v;
              __threadfence_block();
              if (atomicAdd(&ev_cnt[slotr], 1) == 1) {
                __threadfence_block();
                const float tot = ev_part[slotr * 2] + ev_part[slotr * 2 + 1];
                ev_cnt[slotr] = 0;
                const int64_t qb = my_qb;
                const int64_t nvalid =
                    p.n_tokens - qb * 64 < 64 ? p.n_tokens - qb * 64 : 64;
                const int kb = (int)((unsigned)mt >> 12);
                const int j = half ? invB[kb] : invA[kb];
                p.evidence[(slot * p.qb_count + qb) * p.max_blocks + j] = tot / (float)nvalid;
              }
            }
          }
        } else if (ncols < BN) {
          // tail tile: masked columns are -inf, which the MUFU path maps to 0
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            pk[i] = ElemOps<T>::pack2(ex2(fmaf(__uint_as_float(s[2 * i]), c, -mc)),
                                      ex2(fmaf(__uint_as_float(s[2 * i + 1]), c, -mc)));
            publish_done(i + 1);
          }
        } else {
          // full tile: x = s * c - m_ref * c two columns at a time (f32x2
          // FMA); the column pairs selected by kPolyPairs go through the
          // FMA-pipe polynomial, the rest through MUFU, to balance the pipes
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float xa, xb;
            ffma2(xa, xb, __uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]), c, -mc);
            if ((kPolyPairs >> (i & 7)) & 1u)
              pk[i] = exp2_poly_pair<T>(xa, xb);
            else
              pk[i] = exp2_mufu_pair<T>(xa, xb);
            publish_done(i + 1);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) pk[i] = 0u;
#pragma unroll
        for (int hh = 0; hh < P_PARTS; ++hh) publish(hh, pk + PAIRS_PER_PART * hh);
      }
    }

    // ---- epilogue: O / l -> out ----
    if (ok && n_tiles > 0)
      ok = __all_sync(0xffffffffu, tc::mbar_wait(bar(B_OFULL), 0, abort_flag, p.wait_ns));
    tc::tc_fence_after();
    const int64_t qrow = my_qb * 64 + (row & 63);
    const bool valid_row = ok && my_qb >= 0 && qrow < p.n_tokens;
    float l = 0.f;
    if (ok && n_tiles > 0) {
      uint32_t r[8];
      tc::tmem_ld8(t_o + lane_off + 64u, r);
      tc::tmem_wait_ld();
      l = __uint_as_float(r[0]);
    }
    if (p.nsplit > 1) {
      // partial result: O and l relative to 2^(m_ref * c), coalesced by row
      float* part = p.partial + ((w * p.nsplit + split) * 66) * 128;
      const bool have = ok && n_tiles > 0;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t r[32];
        if (have) {
          tc::tmem_ld32(t_o + lane_off + 32u * h2, r);
          tc::tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) part[(h2 * 32 + i) * 128 + row] = __uint_as_float(r[i]);
      }
      part[64 * 128 + row] = have ? l : 0.f;
      part[65 * 128 + row] = (have && has_mass) ? m_ref * c : -INFINITY;
      if (split == 0) p.part_rows[w * 128 + row] = valid_row ? head * p.n_tokens + qrow : -1;
    } else {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T* dst = static_cast<T*>(p.out) + (head * p.n_tokens + qrow) * HD;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      uint32_t r[32];
      if (ok && n_tiles > 0) {
        tc::tmem_ld32(t_o + lane_off + 32u * h2, r);
        tc::tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (valid_row) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 v;
          v.x = ElemOps<T>::pack2(__uint_as_float(r[8 * q4 + 0]) * inv,
                                  __uint_as_float(r[8 * q4 + 1]) * inv);
          v.y = ElemOps<T>::pack2(__uint_as_float(r[8 * q4 + 2]) * inv,
                                  __uint_as_float(r[8 * q4 + 3]) * inv);
          v.z = ElemOps<T>::pack2(__uint_as_float(r[8 * q4 + 4]) * inv,
                                  __uint_as_float(r[8 * q4 + 5]) * inv);
          v.w = ElemOps<T>::pack2(__uint_as_float(r[8 * q4 + 6]) * inv,
                                  __uint_as_float(r[8 * q4 + 7]) * inv);
          reinterpret_cast<uint4*>(dst)[h2 * 4 + q4] = v;
        }
      }
    }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag && p.status) atomicOr(p.status, VGGT_STATUS_TIMEOUT);
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Merges the nsplit partial results of each work item (one CTA per item, one
// thread per row): with M the largest reference max over the splits,
// out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
template <typename T>
__global__ void __launch_bounds__(128)
    combine_splits_kernel(const float* __restrict__ partial, const int64_t* __restrict__ part_rows,
                          int nsplit, T* __restrict__ out) {
  const int64_t item = blockIdx.x;
  const int row = threadIdx.x;
  const int64_t dst = part_rows[item * 128 + row];
  if (dst < 0) return;
  const float* base = partial + item * nsplit * 66 * 128;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, base[(s * 66 + 65) * 128 + row]);
  float acc[64];
#pragma unroll
  for (int d = 0; d < 64; ++d) acc[d] = 0.f;
  float l = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < nsplit; ++s) {
      const float ms = base[(s * 66 + 65) * 128 + row];
      if (ms == -INFINITY) continue;
      const float wgt = exp2f(ms - mx);
      l = fmaf(wgt, base[(s * 66 + 64) * 128 + row], l);
#pragma unroll
      for (int d = 0; d < 64; ++d) acc[d] = fmaf(wgt, base[(s * 66 + d) * 128 + row], acc[d]);
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  uint4* o = reinterpret_cast<uint4*>(out + dst * HD);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint4 v;
    v.x = ElemOps<T>::pack2(acc[8 * q + 0] * inv, acc[8 * q + 1] * inv);
    v.y = ElemOps<T>::pack2(acc[8 * q + 2] * inv, acc[8 * q + 3] * inv);
    v.z = ElemOps<T>::pack2(acc[8 * q + 4] * inv, acc[8 * q + 5] * inv);
    v.w = ElemOps<T>::pack2(acc[8 * q + 6] * inv, acc[8 * q + 7] * inv);
    o[q] = v;
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// [heads, rows, 64] tensor of 2-byte elements, box (64, box_rows, 1), 128-B swizzle.
static bool make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t heads, int64_t rows,
                     uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)rows, (cuuint64_t)heads};
  const cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)rows * HD * 2};
  const cuuint32_t box[3] = {(cuuint32_t)HD, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == VGGT_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace tcattn

bool encode_tmap_3d_sw128(CUtensorMap* map, const void* ptr, int dtype, int64_t d0, int64_t d1,
                          int64_t d2, uint32_t box0, uint32_t box1) {
  tcattn::EncodeTiledFn fn = tcattn::encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  const cuuint64_t strides[2] = {(cuuint64_t)d0 * 2, (cuuint64_t)(d0 * d1) * 2};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == VGGT_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool attn_tc05_supported(const AttnArgs& a) {
  return a.dim == 64 && a.block_q == 64 && a.block_k == 64 && a.n_patch >= 1 &&
         a.scale > 0.f && a.nb <= 65536 && a.max_blocks <= 65536 && a.n_tokens <= 0x7fffffffLL &&
         a.n_patch <= 0x7fffffffLL && a.n_special <= 0x7fffffffLL && a.heads <= 0x7fffffffLL &&
         tcattn::encode_fn() != nullptr;
}

template <typename T, bool EVID>
static cudaError_t launch_kernel(int64_t grid, size_t smem, cudaStream_t stream,
                                 const CUtensorMap& mkp, const CUtensorMap& mvp,
                                 const CUtensorMap& mks, const CUtensorMap& mvs,
                                 const tcattn::Params& p) {
  auto k = tcattn::attn_tc05_kernel<T, EVID>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<(unsigned)grid, tcattn::THREADS, smem, stream>>>(mkp, mvp, mks, mvs, p);
  return cudaGetLastError();
}

cudaError_t launch_combine_splits(const AttnArgs& a, int64_t items, int nsplit,
                                  cudaStream_t stream) {
  if (a.dtype == VGGT_DTYPE_BF16)
    tcattn::combine_splits_kernel<__nv_bfloat16><<<(unsigned)items, 128, 0, stream>>>(
        a.partial, a.part_rows, nsplit, static_cast<__nv_bfloat16*>(a.out));
  else
    tcattn::combine_splits_kernel<__half><<<(unsigned)items, 128, 0, stream>>>(
        a.partial, a.part_rows, nsplit, static_cast<__half*>(a.out));
  return cudaGetLastError();
}

cudaError_t launch_attn_tc05(const AttnArgs& a, cudaStream_t stream) {
  using namespace tcattn;
  if (a.n_slots == 0 || a.qb_count == 0) return cudaSuccess;
  CUtensorMap mkp, mvp, mks, mvs;
  const int64_t ns = a.n_special > 0 ? a.n_special : 1;
  if (!make_map(&mkp, a.pk, a.dtype, a.heads, a.n_patch, BN) ||
      !make_map(&mvp, a.pv, a.dtype, a.heads, a.n_patch, BN) ||
      !make_map(&mks, a.n_special > 0 ? a.sk : a.pk, a.dtype, a.heads,
                a.n_special > 0 ? ns : a.n_patch, BN) ||
      !make_map(&mvs, a.n_special > 0 ? a.sv : a.pv, a.dtype, a.heads,
                a.n_special > 0 ? ns : a.n_patch, BN))
    return cudaErrorInvalidValue;
  Params p;
  p.q = a.q;
  p.indices = a.indices;
  p.counts = a.counts;
  p.head_ids = a.head_ids;
  p.head_dense = a.head_dense;
  p.out = a.out;
  p.status = a.status;
  p.heads = a.heads;
  p.n_tokens = a.n_tokens;
  p.n_patch = a.n_patch;
  p.n_special = a.n_special;
  p.n_slots = a.n_slots;
  p.max_blocks = a.max_blocks;
  p.qb_count = a.qb_count;
  p.nb = a.nb;
  p.pairs = (a.qb_count + 1) / 2;
  p.counts_per_qblock = a.counts_per_qblock;
  p.evidence = a.evidence;
  p.pair_table = a.qblock_pairs;
  p.work_order = a.work_order;
  p.nsplit = a.nsplit > 1 && a.partial != nullptr && a.part_rows != nullptr ? a.nsplit : 1;
  p.partial = a.partial;
  p.part_rows = a.part_rows;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.wait_ns = a.wait_ns > 0 ? a.wait_ns : WAIT_LIMIT_NS;
  p.wait_selftest = a.wait_selftest;
  const bool evid = a.evidence != nullptr;
  const size_t smem = 1024 + OFF_BITMAP + 2 * (size_t)((a.nb + 31) / 32) * 4 +
                      (evid ? 2 * (size_t)((a.nb + 7) & ~7LL) * 2 : 0);
  const int64_t items = a.n_slots * p.pairs;
  const int64_t grid = items * p.nsplit;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  cudaError_t e;
  if (a.dtype == VGGT_DTYPE_BF16)
    e = evid ? launch_kernel<__nv_bfloat16, true>(grid, smem, stream, mkp, mvp, mks, mvs, p)
             : launch_kernel<__nv_bfloat16, false>(grid, smem, stream, mkp, mvp, mks, mvs, p);
  else
    e = evid ? launch_kernel<__half, true>(grid, smem, stream, mkp, mvp, mks, mvs, p)
             : launch_kernel<__half, false>(grid, smem, stream, mkp, mvp, mks, mvs, p);
  if (e != cudaSuccess) return e;
  if (p.nsplit > 1) return launch_combine_splits(a, items, p.nsplit, stream);
  return cudaSuccess;
}

int64_t attn_tc05_split(int64_t items, int sms) {
  // grids of fewer than 4 waves (2 CTAs on each SM) are split toward 8
  // waves, at most 4 ways; longer grids keep one CTA per item
  const int64_t kWave = 2 * (int64_t)(sms > 0 ? sms : 148);
  if (items <= 0 || items >= 4 * kWave) return 1;
  const int64_t s = (8 * kWave + items - 1) / items;
  return s > 4 ? 4 : s;
}

size_t attn_tc05_split_bytes(int64_t items, int64_t nsplit) {
  if (nsplit <= 1) return 0;
  return (((size_t)items * nsplit * 66 * 128 * 4 + 255) & ~(size_t)255) +
         (((size_t)items * 128 * 8 + 255) & ~(size_t)255);
}

}  // namespace vggt
