// Block-sparse attention forward with warp-level mma.sync tiles.
//
// One CTA serves one (query block, slot) pair, the grid of the reference
// kernel (saf3r/triton/adaptive_block_attention.py:78-82).  It walks the
// slot's selected patch blocks (or all of them for a dense-profiled head),
// then the special keys in block_k-sized tiles, with an fp32 online softmax
// (adaptive_block_attention.py:22-58).  K/V tiles are double-buffered with
// cp.async.  Each warp owns 16 query rows.
//
// This kernel covers every shape the reference operator accepts
// (d in {32, 64}, block_q in {32, 64}, block_k in {32, 64, 128}, fp16/bf16)
// and is the reference-shape path; 128-row tcgen05 tiles live in attn_tc05.cu.
#include "common.cuh"
#include "kernels.h"

namespace vggt {

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T>
struct MmaOp;

template <>
struct MmaOp<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

template <>
struct MmaOp<__half> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

struct TileSrc {
  const char* base;  // first element of the head's [rows, D] matrix
  int64_t row0;      // first row of the tile
  int64_t limit;     // rows available in the matrix
  int slot_index;    // evidence slot (-1: none)
  bool valid;
};

}  // namespace

template <typename T, int D, int BQ, int BK, bool EVID>
__global__ void __launch_bounds__(BQ * 2) attn_mma_kernel(AttnArgs a) {
  constexpr int NW = BQ / 16;
  constexpr int NT = NW * 32;
  constexpr int LD = D + 8;  // padded smem row (elements)
  constexpr int CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* qs = reinterpret_cast<T*>(smem_raw);
  T* ks = qs + BQ * LD;       // [2][BK][LD]
  T* vs = ks + 2 * BK * LD;   // [2][BK][LD]
  float* ev_part = reinterpret_cast<float*>(vs + 2 * BK * LD);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int64_t qb = blockIdx.x;
  const int64_t slot = blockIdx.y;
  const int64_t head = a.head_ids[slot];
  if (head < 0 || head >= a.heads) {
    if (tid == 0 && a.status) atomicOr(a.status, VGGT_STATUS_BAD_HEAD);
    return;
  }
  const bool dense = a.head_dense != nullptr && a.head_dense[slot] != 0;
  int64_t count;
  if (dense) {
    count = a.nb;
  } else {
    count = a.counts_per_qblock ? a.counts[slot * a.qb_count + qb] : a.counts[slot];
    if (count < 0 || count > a.max_blocks) {
      if (tid == 0 && a.status) atomicOr(a.status, VGGT_STATUS_BAD_COUNT);
      count = count < 0 ? 0 : a.max_blocks;
    }
  }
  const int64_t n_spec_tiles = (a.n_special + BK - 1) / BK;
  const int64_t total = count + n_spec_tiles;
  const int32_t* row_idx = a.indices + (slot * a.qb_count + qb) * a.max_blocks;
  const size_t esz = sizeof(T);
  const char* pk_head = static_cast<const char*>(a.pk) + head * a.n_patch * D * esz;
  const char* pv_head = static_cast<const char*>(a.pv) + head * a.n_patch * D * esz;
  const char* sk_head = static_cast<const char*>(a.sk) + head * a.n_special * D * esz;
  const char* sv_head = static_cast<const char*>(a.sv) + head * a.n_special * D * esz;
  const int64_t q_row0 = qb * BQ;

  auto tile_src = [&](int64_t t, bool value) -> TileSrc {
    TileSrc s;
    if (t < count) {
      int64_t kb = dense ? t : (int64_t)row_idx[t];
      s.valid = kb >= 0 && kb < a.nb;
      s.base = value ? pv_head : pk_head;
      s.row0 = s.valid ? kb * BK : 0;
      s.limit = a.n_patch;
      s.slot_index = dense ? -1 : (int)t;
    } else {
      const int64_t st = t - count;
      s.valid = true;
      s.base = value ? sv_head : sk_head;
      s.row0 = st * BK;
      s.limit = a.n_special;
      s.slot_index = -1;
    }
    return s;
  };

  auto load_tile = [&](int64_t t, int buf) {
    TileSrc sk = tile_src(t, false);
    TileSrc sv = tile_src(t, true);
    T* kd = ks + buf * BK * LD;
    T* vd = vs + buf * BK * LD;
    for (int i = tid; i < BK * CH; i += NT) {
      const int r = i / CH, ch = i % CH;
      const int64_t gr = sk.row0 + r;
      const bool ok = sk.valid && gr < sk.limit;
      const char* srck = sk.base + ((ok ? gr : 0) * D + ch * 8) * esz;
      const char* srcv = sv.base + ((ok ? gr : 0) * D + ch * 8) * esz;
      cp_async_16(smem_u32(kd + r * LD + ch * 8), srck, ok ? 16 : 0);
      cp_async_16(smem_u32(vd + r * LD + ch * 8), srcv, ok ? 16 : 0);
    }
  };

  // Q tile
  {
    const char* qh = static_cast<const char*>(a.q) + head * a.n_tokens * D * esz;
    for (int i = tid; i < BQ * CH; i += NT) {
      const int r = i / CH, ch = i % CH;
      const int64_t gr = q_row0 + r;
      const bool ok = gr < a.n_tokens;
      cp_async_16(smem_u32(qs + r * LD + ch * 8), qh + ((ok ? gr : 0) * D + ch * 8) * esz,
                  ok ? 16 : 0);
    }
  }
  if (total > 0) load_tile(0, 0);
  cp_async_commit();

  uint32_t qf[D / 16][4];
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = a.scale * kLog2e;
  const int64_t row_a = q_row0 + warp * 16 + g, row_b = row_a + 8;
  const bool va = row_a < a.n_tokens, vb = row_b < a.n_tokens;
  const int nvalid_rows = (int)(a.n_tokens - q_row0 < BQ ? a.n_tokens - q_row0 : BQ);

  for (int64_t t = 0; t < total; ++t) {
    const int buf = (int)(t & 1);
    if (t + 1 < total) {
      load_tile(t + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t addr =
            smem_u32(qs + (warp * 16 + (lane & 15)) * LD + kk * 16 + (lane >> 4) * 8);
        ldsm_x4(addr, qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const TileSrc info = tile_src(t, false);
    if (!info.valid) {
      if (tid == 0 && a.status) atomicOr(a.status, VGGT_STATUS_BAD_INDEX);
      __syncthreads();
      continue;
    }
    const T* kt = ks + buf * BK * LD;
    const T* vt = vs + buf * BK * LD;
    float s[BK / 8][4];
#pragma unroll
    for (int i = 0; i < BK / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < BK / 16; ++np) {
        const int mi = lane >> 3;
        const uint32_t addr =
            smem_u32(kt + (np * 16 + (mi >> 1) * 8 + (lane & 7)) * LD + kk * 16 + (mi & 1) * 8);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        MmaOp<T>::mma(s[2 * np], qf[kk], b0, b1);
        MmaOp<T>::mma(s[2 * np + 1], qf[kk], b2, b3);
      }
    }
    // scale into the log2 domain and mask keys past the end of the matrix
    float lm0 = -INFINITY, lm1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < BK / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t key = info.row0 + nt * 8 + 2 * c + e;
        const bool kv = key < info.limit;
        s[nt][e] = kv ? s[nt][e] * sl2 : -INFINITY;
        s[nt][2 + e] = kv ? s[nt][2 + e] * sl2 : -INFINITY;
        lm0 = fmaxf(lm0, s[nt][e]);
        lm1 = fmaxf(lm1, s[nt][2 + e]);
      }
    }
    lm0 = fmaxf(lm0, __shfl_xor_sync(0xffffffffu, lm0, 1));
    lm0 = fmaxf(lm0, __shfl_xor_sync(0xffffffffu, lm0, 2));
    lm1 = fmaxf(lm1, __shfl_xor_sync(0xffffffffu, lm1, 1));
    lm1 = fmaxf(lm1, __shfl_xor_sync(0xffffffffu, lm1, 2));
    const float nm0 = fmaxf(m0, lm0), nm1 = fmaxf(m1, lm1);
    const float corr0 = fast_exp2(m0 - nm0), corr1 = fast_exp2(m1 - nm1);
    m0 = nm0;
    m1 = nm1;
    float ps0 = 0.f, ps1 = 0.f;
    if constexpr (EVID) {
      // same-pass evidence: the local exponentials feed both the block LSE
      // and the output weights (adaptive_block_attention.py:29-41)
      const float sh0 = fast_exp2(lm0 - nm0), sh1 = fast_exp2(lm1 - nm1);
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < BK / 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x0 = fast_exp2(s[nt][e] - lm0);
          const float x1 = fast_exp2(s[nt][2 + e] - lm1);
          ls0 += x0;
          ls1 += x1;
          s[nt][e] = x0 * sh0;
          s[nt][2 + e] = x1 * sh1;
        }
      }
      ls0 += __shfl_xor_sync(0xffffffffu, ls0, 1);
      ls0 += __shfl_xor_sync(0xffffffffu, ls0, 2);
      ls1 += __shfl_xor_sync(0xffffffffu, ls1, 1);
      ls1 += __shfl_xor_sync(0xffffffffu, ls1, 2);
      if (info.slot_index >= 0) {
        float v = 0.f;
        if (c == 0) {
          if (va) v += (lm0 + __log2f(ls0)) * kLn2;
          if (vb) v += (lm1 + __log2f(ls1)) * kLn2;
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) ev_part[warp] = v;
      }
#pragma unroll
      for (int nt = 0; nt < BK / 8; ++nt) {
        ps0 += s[nt][0] + s[nt][1];
        ps1 += s[nt][2] + s[nt][3];
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < BK / 8; ++nt) {
        s[nt][0] = fast_exp2(s[nt][0] - nm0);
        s[nt][1] = fast_exp2(s[nt][1] - nm0);
        s[nt][2] = fast_exp2(s[nt][2] - nm1);
        s[nt][3] = fast_exp2(s[nt][3] - nm1);
        ps0 += s[nt][0] + s[nt][1];
        ps1 += s[nt][2] + s[nt][3];
      }
    }
    l0 = l0 * corr0 + ps0;
    l1 = l1 * corr1 + ps1;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      o[dt][0] *= corr0;
      o[dt][1] *= corr0;
      o[dt][2] *= corr1;
      o[dt][3] *= corr1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = ElemOps<T>::pack2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = ElemOps<T>::pack2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = ElemOps<T>::pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = ElemOps<T>::pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int mi = lane >> 3;
        const uint32_t addr =
            smem_u32(vt + (kk * 16 + (mi & 1) * 8 + (lane & 7)) * LD + dp * 16 + (mi >> 1) * 8);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(addr, b0, b1, b2, b3);
        MmaOp<T>::mma(o[2 * dp], pa, b0, b1);
        MmaOp<T>::mma(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();
    if constexpr (EVID) {
      if (tid == 0 && info.slot_index >= 0 && a.evidence) {
        float sum = 0.f;
        for (int w = 0; w < NW; ++w) sum += ev_part[w];
        a.evidence[(slot * a.qb_count + qb) * a.max_blocks + info.slot_index] =
            sum / (float)nvalid_rows;
      }
    }
  }

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  T* oh = static_cast<T*>(a.out) + head * a.n_tokens * D;
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    const int col = dt * 8 + 2 * c;
    if (va)
      *reinterpret_cast<uint32_t*>(oh + row_a * D + col) =
          ElemOps<T>::pack2(o[dt][0] * inv0, o[dt][1] * inv0);
    if (vb)
      *reinterpret_cast<uint32_t*>(oh + row_b * D + col) =
          ElemOps<T>::pack2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

template <typename T, int D, int BQ, int BK>
static cudaError_t launch_shape(const AttnArgs& a, cudaStream_t stream) {
  constexpr int LD = D + 8;
  const size_t smem = (size_t)(BQ + 4 * BK) * LD * sizeof(T) + (BQ / 16) * sizeof(float);
  dim3 grid((unsigned)a.qb_count, (unsigned)a.n_slots);
  if (a.evidence) {
    auto k = attn_mma_kernel<T, D, BQ, BK, true>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, BQ * 2, smem, stream>>>(a);
  } else {
    auto k = attn_mma_kernel<T, D, BQ, BK, false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, BQ * 2, smem, stream>>>(a);
  }
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_d(const AttnArgs& a, cudaStream_t s) {
  if (a.block_q == 64) {
    if (a.block_k == 64) return launch_shape<T, D, 64, 64>(a, s);
    if (a.block_k == 128) return launch_shape<T, D, 64, 128>(a, s);
    return launch_shape<T, D, 64, 32>(a, s);
  }
  if (a.block_k == 64) return launch_shape<T, D, 32, 64>(a, s);
  if (a.block_k == 128) return launch_shape<T, D, 32, 128>(a, s);
  return launch_shape<T, D, 32, 32>(a, s);
}

cudaError_t launch_attn_mma(const AttnArgs& a, cudaStream_t s) {
  if (a.n_slots == 0 || a.qb_count == 0) return cudaSuccess;
  if (a.dtype == VGGT_DTYPE_BF16) {
    if (a.dim == 64) return launch_d<__nv_bfloat16, 64>(a, s);
    return launch_d<__nv_bfloat16, 32>(a, s);
  }
  if (a.dim == 64) return launch_d<__half, 64>(a, s);
  return launch_d<__half, 32>(a, s);
}

}  // namespace vggt
