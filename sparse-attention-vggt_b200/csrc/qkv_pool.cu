// QKV projection with the estimator's block pooling in its epilogue.
//
// Computes what saf3r/patch/adaptive_block_value.py:297-315 computes before
// the estimator: qkv = x W^T + b (the module's `qkv` Linear, output rounded
// to the input dtype), q_norm / k_norm (LayerNorm over the 64 dims of a head,
// fp32), RoPE-2D (saf3r/models/official_vggt/layers/rope.py: the first 32
// dims rotate with the token's y position, the last 32 with its x position;
// the caller passes the cos / sin tables), q and k rounded back to the input
// dtype, the token layout's patch / special split
// (saf3r/patch/value_evolving_attention.py:17-20), and the block means the
// estimator pools (adaptive_block_value.py:16-23 block_mean) over 64-token
// query blocks of q and 64-row blocks of the patch keys.
//
// One work tile = 128 token rows x one head: a tcgen05 GEMM of M=128, N=192
// (the head's 64 q, 64 k and 64 v rows of W, three TMA boxes per K step),
// K = model dim in steps of 64 through a 3-stage TMA ring, fp32 accumulator
// in TMEM.  CTAs are persistent (one per SM) with two TMEM accumulators and
// two epilogue warpgroups (warps 4-7 and 8-11, one token row per thread)
// that take alternate tiles, so two tiles' epilogues run at once (two warps
// per SM sub-partition to hide each other's latencies) while the MMAs of the
// next tile proceed.  setmaxnreg moves registers from the producer / MMA
// warpgroup to the epilogue warpgroups.  A thread holds a whole head row, so
// LayerNorm and RoPE need no cross-thread traffic; block sums go through a
// shared-memory transpose in a fixed order (deterministic).  Query blocks
// never straddle tiles (128 = 2 x 64 rows); patch-key blocks can, so each
// tile writes its partial sums of the (at most three) patch blocks it
// touches and a second, small kernel folds a block's partials in tile order.
//
// Every wait is bounded (1 s); on expiry the CTA raises an abort flag, sets
// VGGT_STATUS_TIMEOUT, drains its copies and MMAs, frees TMEM and exits.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace vggt {

namespace qkvp {

constexpr int BM = 128;     // token rows per tile
constexpr int HD = 64;      // head dim
constexpr int BK = 64;      // K per stage
constexpr int NO = 3 * HD;  // MMA N: q | k | v of one head
constexpr int NST = 3;
// warpgroup 0: TMA producer (warp 0), MMA issuer (warp 1), two idle warps;
// warpgroups 1 and 2: the epilogue, on alternating tiles (accumulator i % 2)
constexpr int THREADS = 384;
// register split (setmaxnreg): the launch gives every thread LAUNCH_REGS;
// warpgroup 0 gives back down to CTRL_REGS and the two epilogue warpgroups
// take the difference: 128 * CTRL_REGS + 256 * EPI_REGS = 384 * LAUNCH_REGS
constexpr int LAUNCH_REGS = 168;
constexpr int CTRL_REGS = 56;
constexpr int EPI_REGS = 224;
static_assert(128 * CTRL_REGS + 256 * EPI_REGS == THREADS * LAUNCH_REGS, "register split");
constexpr uint32_t A_BYTES = BM * BK * 2;  // 16 KB
constexpr uint32_t B_BYTES = NO * BK * 2;  // 24 KB
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t TMEM_COLS = 512;        // two accumulators of 192 in 256-column slots
constexpr uint64_t LIMIT_NS = 1000000000ull;
constexpr int TPITCH = HD + 1;             // transpose buffer row pitch (floats)

constexpr uint32_t OFF_STAGE = 0;
constexpr uint32_t OFF_T = NST * STAGE_BYTES;              // float[2 groups][BM][TPITCH]
constexpr uint32_t OFF_KINFO = OFF_T + 2 * BM * TPITCH * 4;  // int[2][4 warps][4]: block boundaries
constexpr uint32_t OFF_KX = OFF_KINFO + 2 * 4 * 4 * 4;     // float[2][3][64]: half-1 key partials
constexpr uint32_t OFF_LN = OFF_KX + 2 * 3 * HD * 4;       // float[4][64]: q_norm w, b, k_norm w, b
constexpr uint32_t OFF_BAR = OFF_LN + 4 * HD * 4;
constexpr int B_FULL = 0;                 // [NST]
constexpr int B_EMPTY = B_FULL + NST;     // [NST]
constexpr int B_ACCFULL = B_EMPTY + NST;  // [2]
constexpr int B_ACCEMPTY = B_ACCFULL + 2; // [2]
constexpr int B_DRAIN = B_ACCEMPTY + 2;
constexpr int NBAR = B_DRAIN + 1;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;           // tmem base, abort flag, votes
constexpr uint32_t OFF_ROPE = (OFF_MISC + 128 + 15) & ~15u;  // float2[pos_count][16] (cos, sin)

struct Params {
  const void* bias;     // [3C] in x's dtype, or null
  const float* qn_w;    // [64] LayerNorm weight / bias of q, or null (no q_norm)
  const float* qn_b;
  const float* kn_w;    // [64] of k, or null
  const float* kn_b;
  const int32_t* pos;   // [N, 2] (y, x) token positions, or null (no RoPE)
  const float* rope_cos;  // [pos_count, 16]
  const float* rope_sin;
  void* q;              // [H, N, 64]
  void* kp;             // [H, NP, 64]
  void* vp;
  void* ks;             // [H, NS, 64]
  void* vs;
  float* pooled_q;      // [H, QB, 64] means, or null
  float* part_k;        // [row tiles, H, 3, 64] partial sums of patch-key blocks, or null
  int32_t* part_blk;    // [row tiles, H, 3] their block ids (-1 unused)
  int32_t* status;
  int64_t n, n_patch, n_special, qb_count;
  int heads, k_steps;   // model dim / 64
  int tok_per_frame, special_per_frame;
  int pos_count;        // rows of the RoPE tables (largest position + 1)
  int bias_smem;        // 1: the bias is staged in shared memory as fp32 (after the RoPE table)
  float ln_eps;
  int64_t tiles;        // row tiles x heads
};

__device__ __forceinline__ float elem_to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float elem_to_float(__half x) { return __half2float(x); }

// patch index of a token, or -1 for a special token (token counts stay
// below 2^31, which the host checks, so 32-bit unsigned division suffices)
__device__ __forceinline__ int patch_of(uint32_t t, const Params& p) {
  const uint32_t tpf = (uint32_t)p.tok_per_frame, spf = (uint32_t)p.special_per_frame;
  const uint32_t f = t / tpf;
  const uint32_t j = t - f * tpf;
  if (j < spf) return -1;
  return (int)(f * (tpf - spf) + (j - spf));
}

// rounds 64 values to the element type: packed words w[32] (what is stored)
// and, when `back` is set, the rounded values back in v
template <typename T>
__device__ __forceinline__ void round_pack(float* v, uint32_t* w, bool back) {
#pragma unroll
  for (int i = 0; i < HD / 2; ++i) {
    w[i] = ElemOps<T>::pack2(v[2 * i], v[2 * i + 1]);
    if (back) {
      const float2 f = ElemOps<T>::to_float2(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

// LayerNorm (biased variance, like torch.nn.LayerNorm) and RoPE-2D of one
// head row held by the thread.  The rotation is x cos + rotate(x) sin with
// rotate(a, b) = (-b, a) over each 32-dim half, as separately rounded fp32
// products and sum.
__device__ __forceinline__ void norm_rope(float* v, const float* w, const float* b, float eps,
                                          bool rope, int py, int px, const float2* table) {
  if (w != nullptr) {
    // eight interleaved partial sums keep the dependent chains short
    float s8[8], q8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s8[j] = 0.f;
#pragma unroll
    for (int i = 0; i < HD; ++i) s8[i & 7] += v[i];
    const float mean =
        (((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]))) * (1.f / HD);
#pragma unroll
    for (int j = 0; j < 8; ++j) q8[j] = 0.f;
#pragma unroll
    for (int i = 0; i < HD; ++i) {
      v[i] -= mean;  // centred once, reused below
      q8[i & 7] = fmaf(v[i], v[i], q8[i & 7]);
    }
    const float q =
        ((q8[0] + q8[1]) + (q8[2] + q8[3])) + ((q8[4] + q8[5]) + (q8[6] + q8[7]));
    const float rstd = rsqrtf(q * (1.f / HD) + eps);
    // w and b are shared-memory copies of the LayerNorm parameters
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int i = 0; i < HD / 4; ++i) {
      const float4 ww = w4[i], bb = b4[i];
      v[4 * i + 0] = fmaf(v[4 * i + 0] * rstd, ww.x, bb.x);
      v[4 * i + 1] = fmaf(v[4 * i + 1] * rstd, ww.y, bb.y);
      v[4 * i + 2] = fmaf(v[4 * i + 2] * rstd, ww.z, bb.z);
      v[4 * i + 3] = fmaf(v[4 * i + 3] * rstd, ww.w, bb.w);
    }
  }
  if (rope) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const float2* cs = table + (half ? px : py) * 16;
      float* u = v + 32 * half;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 c = cs[i];
        const float a = u[i], bb = u[i + 16];
        u[i] = __fadd_rn(__fmul_rn(a, c.x), __fmul_rn(-bb, c.y));
        u[i + 16] = __fadd_rn(__fmul_rn(bb, c.x), __fmul_rn(a, c.y));
      }
    }
  }
}

// the 128 threads of epilogue group g (named barrier 1 + g)
__device__ __forceinline__ void epi_sync(int g) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory");
}

template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// 64 consecutive packed values (32 words) as 8 16-byte stores
template <typename T>
__device__ __forceinline__ void store_row(T* dst, const uint32_t* w) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 8; ++q) d[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1)
    qkv_pool_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w, Params p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw_addr);
  const uint32_t bar0 = base + OFF_BAR;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(sbase + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  float* tbuf = reinterpret_cast<float*>(sbase + OFF_T);
  float2* table = reinterpret_cast<float2*>(sbase + OFF_ROPE);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t H = p.heads;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(bar(B_FULL + s), 1);
      tc::mbar_init(bar(B_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar(B_ACCFULL + b), 1);
      tc::mbar_init(bar(B_ACCEMPTY + b), 128);
    }
    tc::mbar_init(bar(B_DRAIN), 1);
    misc[1] = 0u;
    tc::mbar_fence_init();
  }
  if (p.pos != nullptr)
    for (int e = tid; e < p.pos_count * 16; e += THREADS)
      table[e] = make_float2(p.rope_cos[e], p.rope_sin[e]);
  if (p.bias_smem) {
    // the whole bias vector [3C] as fp32, after the RoPE table
    float* bs = reinterpret_cast<float*>(sbase + OFF_ROPE) + p.pos_count * 32;
    const T* bsrc = static_cast<const T*>(p.bias);
    for (int e = tid; e < 3 * p.heads * HD; e += THREADS) bs[e] = elem_to_float(bsrc[e]);
  }
  float* ln = reinterpret_cast<float*>(sbase + OFF_LN);  // q_norm w, b, k_norm w, b
  if (tid < 4 * HD) {
    const float* src[4] = {p.qn_w, p.qn_b, p.kn_w, p.kn_b};
    const float* sp = src[tid / HD];
    ln[tid] = sp != nullptr ? sp[tid % HD] : 0.f;
  }
  if (warp == 1) {
    tc::tmem_alloc(base + OFF_MISC, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = misc[0];

  // each warpgroup sets its register share at the top of its own branch:
  // warpgroup 0 gives registers back, the epilogue warpgroups take them
  if (warp < 4) regs_dec<CTRL_REGS>();
  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      tc::prefetch_tmap(&tm_x);
      tc::prefetch_tmap(&tm_w);
      int64_t it = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; ok && u < p.tiles; u += gridDim.x) {
        const int rt = (int)(u / H), h = (int)(u % H);
        for (int k = 0; k < p.k_steps; ++k, ++it) {
          const int s = (int)(it % NST);
          if (it >= NST &&
              !tc::mbar_wait(bar(B_EMPTY + s), (uint32_t)((it / NST - 1) & 1), abort_flag,
                             LIMIT_NS)) {
            ok = false;
            break;
          }
          const uint32_t dst = base + OFF_STAGE + (uint32_t)s * STAGE_BYTES;
          tc::mbar_expect_tx(bar(B_FULL + s), STAGE_BYTES);
          tc::tma_load_3d(dst, &tm_x, bar(B_FULL + s), k * BK, rt * BM, 0);
          const int c = p.heads * HD;  // model dim
#pragma unroll
          for (int j = 0; j < 3; ++j)
            tc::tma_load_3d(dst + A_BYTES + (uint32_t)j * (HD * BK * 2), &tm_w, bar(B_FULL + s),
                            k * BK, j * c + h * HD, 0);
        }
      }
      // drain: the last NST stages' copies, landed or not
      for (int64_t t = it > NST ? it - NST : 0; t < it; ++t)
        tc::mbar_wait_drain(bar(B_FULL + (int)(t % NST)), (uint32_t)((t / NST) & 1), LIMIT_NS);
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc = tc::idesc_f16(fmt, 0u, BM, NO);
      int64_t it = 0, i = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; ok && u < p.tiles; u += gridDim.x, ++i) {
        const int b = (int)(i & 1);
        // the epilogue must have read accumulator b (tile i - 2) out
        if (i >= 2 && !tc::mbar_wait(bar(B_ACCEMPTY + b), (uint32_t)(((i >> 1) + 1) & 1),
                                     abort_flag, LIMIT_NS)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)b * 256u;
        for (int k = 0; k < p.k_steps; ++k, ++it) {
          const int s = (int)(it % NST);
          if (!tc::mbar_wait(bar(B_FULL + s), (uint32_t)((it / NST) & 1), abort_flag, LIMIT_NS)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_addr = base + OFF_STAGE + (uint32_t)s * STAGE_BYTES;
          const uint64_t adesc = tc::sw128_desc(a_addr, 16);
          const uint64_t bdesc = tc::sw128_desc(a_addr + A_BYTES, 16);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc::mma_ss(acc, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2), idesc,
                       (k > 0 || kk > 0) ? 1u : 0u);
          tc::mma_commit(bar(B_EMPTY + s));
        }
        if (ok) tc::mma_commit(bar(B_ACCFULL + b));
      }
      tc::mma_commit(bar(B_DRAIN));
      tc::mbar_wait_drain(bar(B_DRAIN), 0, LIMIT_NS);
    }
  } else if (warp >= 4) {
    regs_inc<EPI_REGS>();
    // ====== epilogue: groups of warps 4-7 and 8-11, one token row per thread ======
    // group g takes the CTA's tiles i = g, g + 2, ... (accumulator g)
    const int g = (warp - 4) >> 2;
    const int sub = warp & 3;          // TMEM lane quarter of this warp
    const int row = sub * 32 + lane;   // 0..127
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const bool rope = p.pos != nullptr;
    float* tb = tbuf + g * BM * TPITCH;
    int* kinfo = reinterpret_cast<int*>(sbase + OFF_KINFO) + g * 16;
    // one flag per warp, double-buffered by tile so that a tile's votes are
    // read before the group's next-but-one tile overwrites them
    volatile int* vote0 = reinterpret_cast<volatile int*>(misc + 8 + 8 * g);
    float* kx = reinterpret_cast<float*>(sbase + OFF_KX) + g * 3 * HD;
    const T* bias = static_cast<const T*>(p.bias);
    const bool bias16 = (reinterpret_cast<uintptr_t>(bias) & 15u) == 0;
    const float* bias_s =
        p.bias_smem ? reinterpret_cast<const float*>(sbase + OFF_ROPE) + p.pos_count * 32 : nullptr;
    for (int64_t i = g;; i += 2) {
      const int64_t u = blockIdx.x + i * gridDim.x;
      if (u >= p.tiles) break;
      const int b = g;  // == i & 1
      const int rt = (int)(u / H);
      const int h = (int)(u % H);
      const uint32_t t = (uint32_t)rt * BM + row;
      const bool valid = t < (uint64_t)p.n;
      // token positions do not depend on the accumulator: load them first
      int py = 0, px = 0;
      if (rope && valid) {
        py = p.pos[2 * t];
        px = p.pos[2 * t + 1];
      }
      const bool got = tc::mbar_wait(bar(B_ACCFULL + b), (uint32_t)((i >> 1) & 1), abort_flag,
                                     LIMIT_NS);
      // the group's four warps leave together (the named barriers below are
      // not bounded, so no warp may stop at one the others never reach)
      const bool warp_ok = __all_sync(0xffffffffu, got);
      volatile int* vote = vote0 + 4 * (int)((i >> 1) & 1);
      if (lane == 0) vote[sub] = warp_ok ? 1 : 0;
      epi_sync(g);
      const bool all_ok = vote[0] && vote[1] && vote[2] && vote[3];
      if (!all_ok) break;
      tc::tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)b * 256u + lane_off;
      const int pidx = valid ? patch_of(t, p) : -1;
      py = py < 0 ? 0 : (py >= p.pos_count ? p.pos_count - 1 : py);
      px = px < 0 ? 0 : (px >= p.pos_count ? p.pos_count - 1 : px);
      // part j's 64 accumulator columns arrive in r while part j-1 is processed
      uint32_t r[64];
      tc::tmem_ld32(acc, r);
      tc::tmem_ld32(acc + 32u, r + 32);
      tc::tmem_wait_ld();
      float v[HD];
      uint32_t w[HD / 2];
#pragma unroll 1
      for (int part = 0; part < 3; ++part) {
        // accumulator columns [64 part, 64 part + 64): q, k, v of head h
#pragma unroll
        for (int d = 0; d < HD; ++d) v[d] = __uint_as_float(r[d]);
        if (part < 2) {
          tc::tmem_ld32(acc + (uint32_t)(64 * part + 64), r);
          tc::tmem_ld32(acc + (uint32_t)(64 * part + 96), r + 32);
        }
        const int bcol = part * p.heads * HD + h * HD;
        if (bias_s != nullptr) {
          const float4* b4 = reinterpret_cast<const float4*>(bias_s + bcol);
#pragma unroll
          for (int q = 0; q < HD / 4; ++q) {
            const float4 bb = b4[q];
            v[4 * q] += bb.x;
            v[4 * q + 1] += bb.y;
            v[4 * q + 2] += bb.z;
            v[4 * q + 3] += bb.w;
          }
        } else if (bias != nullptr) {
          if (bias16) {
            const uint4* b4 = reinterpret_cast<const uint4*>(bias + bcol);
#pragma unroll
            for (int q = 0; q < HD / 8; ++q) {
              const uint4 w4 = __ldg(b4 + q);
              const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 bb = ElemOps<T>::to_float2(wv[e]);
                v[8 * q + 2 * e] += bb.x;
                v[8 * q + 2 * e + 1] += bb.y;
              }
            }
          } else {
#pragma unroll
            for (int d = 0; d < HD; ++d) v[d] += elem_to_float(bias[bcol + d]);
          }
        }
        // the Linear's output is rounded to the activation dtype
        round_pack<T>(v, w, part < 2);
        if (part < 2) {
          const bool has_norm = (part == 0 ? p.qn_w : p.kn_w) != nullptr;
          norm_rope(v, has_norm ? ln + 2 * part * HD : nullptr, ln + (2 * part + 1) * HD,
                    p.ln_eps, rope, py, px, table);
          round_pack<T>(v, w, true);
        }
        if (valid) {
          T* dst;
          if (part == 0) {
            dst = static_cast<T*>(p.q) + ((int64_t)h * p.n + t) * HD;
          } else if (pidx >= 0) {
            dst = static_cast<T*>(part == 1 ? p.kp : p.vp) + ((int64_t)h * p.n_patch + pidx) * HD;
          } else {
            const uint32_t f = t / (uint32_t)p.tok_per_frame;
            const uint32_t sidx = f * (uint32_t)p.special_per_frame + (t - f * (uint32_t)p.tok_per_frame);
            dst = static_cast<T*>(part == 1 ? p.ks : p.vs) + ((int64_t)h * p.n_special + sidx) * HD;
          }
          store_row<T>(dst, w);
        }
        if (part < 2) {
          tc::tmem_wait_ld();  // part + 1 is in r
          if (part == 1) {
            // the accumulator is read out: the next tile's MMAs may start
            tc::tc_fence_before();
            tc::mbar_arrive(bar(B_ACCEMPTY + b));
          }
        }
        if (part == 0 && p.pooled_q != nullptr) {
          // query-block means: thread (half, col) sums column col over rows
          // [64 half, 64 half + 64) of the tile (four interleaved partial sums)
#pragma unroll
          for (int d = 0; d < HD; ++d) tb[row * TPITCH + d] = valid ? v[d] : 0.f;
          epi_sync(g);
          const int half = row >> 6, col = row & 63;
          const int64_t qb = rt * 2 + half;
          if (qb < p.qb_count) {
            float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
            for (int j = 0; j < 64; ++j) a[j & 3] += tb[(half * 64 + j) * TPITCH + col];
            const int64_t nrow = p.n - qb * 64 < 64 ? p.n - qb * 64 : 64;
            p.pooled_q[(h * p.qb_count + qb) * HD + col] =
                ((a[0] + a[1]) + (a[2] + a[3])) / (float)nrow;
          }
          epi_sync(g);
        }
        if (part == 1 && p.part_k != nullptr) {
          // patch-key block partial sums over this tile's patch rows.  The tile
          // touches blocks first .. first + 2 at most (128 patch rows), in
          // nondecreasing order down the rows; special and invalid rows hold
          // zeros.  So slot s covers the row range [start_s, start_{s+1}) with
          // start_s the first row whose block slot is >= s, and thread (half,
          // col) sums column col of its half's rows range by range; the halves
          // are then added (half 0 + half 1).
          int first = -1;
          {
            const uint32_t t0 = (uint32_t)rt * BM, tpf = (uint32_t)p.tok_per_frame;
            const uint32_t f = t0 / tpf, j = t0 - f * tpf;
            const uint32_t tf = j < (uint32_t)p.special_per_frame
                                    ? f * tpf + (uint32_t)p.special_per_frame
                                    : t0;
            if (tf < (uint64_t)p.n && tf < t0 + BM) first = patch_of(tf, p) >> 6;
          }
#pragma unroll
          for (int d = 0; d < HD; ++d) tb[row * TPITCH + d] = pidx >= 0 ? v[d] : 0.f;
          const int sl = pidx >= 0 ? (int)(pidx >> 6) - first : -1;  // slot 0..2, -1 none
          {
            // per warp: the first row with slot >= 1 and >= 2, and which
            // slots occur
            const unsigned ge1 = __ballot_sync(0xffffffffu, sl >= 1);
            const unsigned ge2 = __ballot_sync(0xffffffffu, sl >= 2);
            const unsigned s0 = __ballot_sync(0xffffffffu, sl == 0);
            const unsigned s1 = __ballot_sync(0xffffffffu, sl == 1);
            if (lane == 0) {
              kinfo[sub * 4 + 0] = ge1 ? sub * 32 + __ffs(ge1) - 1 : BM;
              kinfo[sub * 4 + 1] = ge2 ? sub * 32 + __ffs(ge2) - 1 : BM;
              kinfo[sub * 4 + 2] = (s0 ? 1 : 0) | (s1 ? 2 : 0) | (ge2 ? 4 : 0);
            }
          }
          epi_sync(g);
          int start1 = BM, start2 = BM, seen = 0;
#pragma unroll
          for (int w2 = 0; w2 < 4; ++w2) {
            start1 = min(start1, kinfo[w2 * 4 + 0]);
            start2 = min(start2, kinfo[w2 * 4 + 1]);
            seen |= kinfo[w2 * 4 + 2];
          }
          const int half = row >> 6, col = row & 63;
          const int lo = half * 64, hi = lo + 64;
          auto range_sum = [&](int j0, int j1) {
            j0 = j0 < lo ? lo : (j0 > hi ? hi : j0);
            j1 = j1 < lo ? lo : (j1 > hi ? hi : j1);
            float x0 = 0.f, x1 = 0.f;
            int j = j0;
            for (; j + 1 < j1; j += 2) {
              x0 += tb[j * TPITCH + col];
              x1 += tb[(j + 1) * TPITCH + col];
            }
            if (j < j1) x0 += tb[j * TPITCH + col];
            return x0 + x1;
          };
          const float a0 = range_sum(0, start1);
          const float a1 = range_sum(start1, start2);
          const float a2 = range_sum(start2, BM);
          if (half == 1) {
            kx[col] = a0;
            kx[64 + col] = a1;
            kx[128 + col] = a2;
          }
          epi_sync(g);
          if (half == 0) {
            const int64_t pbase = (rt * H + h) * 3;
            p.part_k[(pbase + 0) * HD + col] = a0 + kx[col];
            p.part_k[(pbase + 1) * HD + col] = a1 + kx[64 + col];
            p.part_k[(pbase + 2) * HD + col] = a2 + kx[128 + col];
            if (col < 3) p.part_blk[pbase + col] = (seen >> col) & 1 ? first + col : -1;
          }
          // no barrier here: tb is next written after the next tile's vote
          // barrier, and kx after two more of this group's barriers
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

// Patch-key block means from the tiles' partial sums: one warp per (head,
// block), the block's (at most two) tiles added in tile order.
__global__ void __launch_bounds__(256)
    fold_k_kernel(const float* __restrict__ part_k, const int32_t* __restrict__ part_blk,
                  int64_t heads, int64_t nb, int64_t n_patch, int tok_per_frame,
                  int special_per_frame, float* __restrict__ pooled_k) {
  const int lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (unit >= heads * nb) return;
  const int64_t h = unit / nb, blk = unit % nb;
  const int ppf = tok_per_frame - special_per_frame;
  auto token_of = [&](int64_t pi) {
    return (pi / ppf) * tok_per_frame + special_per_frame + pi % ppf;
  };
  const int64_t p0 = blk * 64;
  const int64_t p1 = (blk + 1) * 64 < n_patch ? (blk + 1) * 64 - 1 : n_patch - 1;
  const int64_t t_lo = token_of(p0) / BM, t_hi = token_of(p1) / BM;
  float s0 = 0.f, s1 = 0.f;
  for (int64_t rt = t_lo; rt <= t_hi; ++rt) {
    const int64_t pbase = (rt * heads + h) * 3;
    for (int sl = 0; sl < 3; ++sl)
      if (part_blk[pbase + sl] == blk) {
        s0 += part_k[(pbase + sl) * HD + lane];
        s1 += part_k[(pbase + sl) * HD + lane + 32];
      }
  }
  const float pop = (float)(p1 - p0 + 1);
  pooled_k[(h * nb + blk) * HD + lane] = s0 / pop;
  pooled_k[(h * nb + blk) * HD + lane + 32] = s1 / pop;
}

static size_t smem_bytes(int pos_count) {
  return 1024 + OFF_ROPE + (size_t)pos_count * 16 * sizeof(float2);
}
// with the bias staged in shared memory (fp32, 3C values)
static size_t smem_bytes_bias(int pos_count, int heads) {
  return smem_bytes(pos_count) + (size_t)3 * heads * HD * 4;
}

}  // namespace qkvp

size_t qkv_pool_partial_bytes(int64_t n_tokens, int heads) {
  const int64_t rt = (n_tokens + qkvp::BM - 1) / qkvp::BM;
  return (((size_t)rt * heads * 3 * qkvp::HD * 4 + 255) & ~(size_t)255) +
         (((size_t)rt * heads * 3 * 4 + 255) & ~(size_t)255);
}

bool qkv_pool_supported(int pos_count) {
  return pos_count >= 0 && qkvp::smem_bytes(pos_count) <= 227u * 1024u;
}

cudaError_t launch_qkv_pool(const QkvPoolArgs& a, cudaStream_t stream) {
  using namespace qkvp;
  if (a.n_tokens == 0) return cudaSuccess;
  const int c = a.heads * HD;
  CUtensorMap mx, mw;
  if (!encode_tmap_3d_sw128(&mx, a.x, a.dtype, c, a.n_tokens, 1, BK, BM) ||
      !encode_tmap_3d_sw128(&mw, a.w, a.dtype, c, 3 * c, 1, BK, HD))
    return cudaErrorInvalidValue;
  Params p;
  p.bias = a.bias;
  p.qn_w = a.qn_w;
  p.qn_b = a.qn_b;
  p.kn_w = a.kn_w;
  p.kn_b = a.kn_b;
  p.pos = a.pos;
  p.rope_cos = a.rope_cos;
  p.rope_sin = a.rope_sin;
  p.q = a.q;
  p.kp = a.kp;
  p.vp = a.vp;
  p.ks = a.ks;
  p.vs = a.vs;
  p.pooled_q = a.pooled_q;
  p.status = a.status;
  p.n = a.n_tokens;
  p.tok_per_frame = a.tok_per_frame;
  p.special_per_frame = a.special_per_frame;
  const int64_t frames = a.n_tokens / a.tok_per_frame;
  p.n_patch = frames * (a.tok_per_frame - a.special_per_frame);
  p.n_special = frames * a.special_per_frame;
  p.qb_count = (a.n_tokens + 63) / 64;
  p.heads = a.heads;
  p.k_steps = c / BK;
  p.pos_count = a.pos != nullptr ? a.pos_count : 0;
  p.ln_eps = a.ln_eps;
  const int64_t rtiles = (a.n_tokens + BM - 1) / BM;
  p.tiles = rtiles * a.heads;
  unsigned char* ws = static_cast<unsigned char*>(a.workspace);
  p.part_k = a.pooled_k != nullptr ? reinterpret_cast<float*>(ws) : nullptr;
  p.part_blk = a.pooled_k != nullptr
                   ? reinterpret_cast<int32_t*>(
                         ws + (((size_t)rtiles * a.heads * 3 * HD * 4 + 255) & ~(size_t)255))
                   : nullptr;
  p.bias_smem = a.bias != nullptr && smem_bytes_bias(p.pos_count, a.heads) <= 227u * 1024u;
  const size_t smem = p.bias_smem ? smem_bytes_bias(p.pos_count, a.heads) : smem_bytes(p.pos_count);
  int sms = 0, dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int64_t grid = p.tiles < sms ? p.tiles : sms;
  // The register split assumes LAUNCH_REGS per thread at launch; with any
  // other count the epilogue's setmaxnreg.inc could never be satisfied, so
  // such a build does not launch at all.
  auto launch = [&](auto k) -> cudaError_t {
    cudaFuncAttributes fa;
    cudaError_t r = cudaFuncGetAttributes(&fa, k);
    if (r != cudaSuccess) return r;
    if (fa.numRegs != LAUNCH_REGS) return cudaErrorInvalidConfiguration;
    r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (r != cudaSuccess) return r;
    k<<<(unsigned)grid, THREADS, smem, stream>>>(mx, mw, p);
    return cudaSuccess;
  };
  e = a.dtype == VGGT_DTYPE_BF16 ? launch(qkv_pool_kernel<__nv_bfloat16>)
                                 : launch(qkv_pool_kernel<__half>);
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (e != cudaSuccess || a.pooled_k == nullptr) return e;
  const int64_t nb = (p.n_patch + 63) / 64;
  const int64_t units = a.heads * nb;
  fold_k_kernel<<<(unsigned)((units + 7) / 8), 256, 0, stream>>>(
      p.part_k, p.part_blk, a.heads, nb, p.n_patch, a.tok_per_frame, a.special_per_frame,
      a.pooled_k);
  return cudaGetLastError();
}

}  // namespace vggt
