// Per-token sparse attention: every query attends to its own list of keys.
//
// Computes what saf3r/triton/sparse_topk_attention.py:115-166
// (fused_sparse_topk_attention) and :261-286 (its online-softmax variant)
// compute: out[n] = softmax_j(q_n . k[idx[n, j]] * scale) . v[idx[n, j]], fp32
// softmax and accumulation, any top-k length.  Each query has its own key set,
// so there is no shared tile for the tensor cores: this is a gather workload,
// bound by L2 (a head's K/V stay L2-resident) rather than by math.
//
// One warp per query, keys in chunks of 32 with an online softmax in the exp2
// domain:
//   * scores: the chunk's K rows are gathered coalesced (D/8 lanes per row, a
//     16-byte segment each), dotted segment-wise with the query, summed across
//     the row's lanes, and key idx[c + j]'s score is moved to lane j;
//   * P.V: each half-warp takes one key at a time, its 16 lanes holding D/16
//     dims each, so every gathered V row is read as one coalesced segment;
//     the two halves' sums combine at the end.
// All of a chunk's gathers are issued before their first use (the kernel is
// bound by L2 latency otherwise), with selects instead of branches.
// Index entries outside [0, n_keys) are skipped and reported as
// VGGT_STATUS_BAD_INDEX (the reference reads them unchecked).
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace vggt {

namespace tokattn {

constexpr int WARPS = kTokenAttnQueriesPerCta;  // queries per CTA (3 CTAs per SM at dim 64)

template <int N>
struct Vec;  // N bf16/fp16 values as one load
template <>
struct Vec<2> {
  using type = uint32_t;
};
template <>
struct Vec<4> {
  using type = uint2;
};
template <>
struct Vec<8> {
  using type = uint4;
};

template <typename T, int N>
__device__ __forceinline__ void unpack(const typename Vec<N>::type& raw, float* f) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const float2 x = ElemOps<T>::to_float2(w[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(WARPS * 32, 4)
    token_attn_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                      const int32_t* __restrict__ idx, int64_t idx_stride, int64_t n_queries,
                      int64_t n_keys, int64_t topk, float scale_log2, T* __restrict__ out,
                      int32_t* status) {
  constexpr int PD = D / 16;  // V dims per lane in the P.V phase
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  const int64_t r = (int64_t)blockIdx.x * WARPS + warp;
  if (r >= n_queries) return;

  // K rows are read whole and coalesced: SEG lanes share a row, each holding
  // one 16-byte segment (8 elements), so one load instruction covers RPI rows
  // (a lane reading a whole row by itself costs an L1 wavefront per row per
  // instruction, which bounded the gather).  Each lane keeps its segment of
  // the query row, fp32.
  constexpr int SEG = D / 8, RPI = 32 / SEG;
  const int grp = lane / SEG, seg = lane % SEG;
  float q8[8];
  {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(q + r * D) + seg);
    unpack<T, 8>(raw, q8);
  }
  const int half = lane >> 4;     // which key of a pair this half-warp takes
  const int dim0 = (lane & 15) * PD;
  float acc[PD];
#pragma unroll
  for (int i = 0; i < PD; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool bad = false;
  const int32_t* irow = idx + r * idx_stride;

  // V slices fetched per group before they are used: all 16 of a chunk for
  // dims up to 64, 4 at a time for 128 (register budget)
  constexpr int G = D <= 64 ? 16 : 4;
  using VT = typename Vec<PD>::type;
  // each chunk's key index is loaded one chunk ahead
  int32_t kb_next = lane < topk ? irow[lane] : -1;
  for (int64_t c = 0; c < topk; c += 32) {
    const int64_t j = c + lane;
    const bool in_range = j < topk;
    const int32_t kb = in_range ? kb_next : -1;
    if (j + 32 < topk) kb_next = irow[j + 32];
    const bool ok = in_range && kb >= 0 && kb < n_keys;
    bad |= in_range && !ok;
    // every gather of the chunk is issued before any of it is used: this
    // lane's segment of keys RPI*i + grp (i < SEG), then the first group of
    // V slices of its half-warp's keys
    uint4 kraw[SEG];
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const int src = RPI * i + grp;
      const int32_t ki = __shfl_sync(full, kb, src);
      const bool oki = c + src < topk && ki >= 0 && ki < n_keys;
      kraw[i] = __ldg(reinterpret_cast<const uint4*>(k + (int64_t)(oki ? ki : 0) * D) + seg);
    }
    VT vraw[G];
    bool vok[G];
    auto fetch_v = [&](int g0) {
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        const int src = 2 * (g0 + gi) + half;
        const int32_t ik = __shfl_sync(full, kb, src);
        const bool okk = __shfl_sync(full, (int)ok, src) != 0;
        vraw[gi] = *reinterpret_cast<const VT*>(v + (int64_t)(okk ? ik : 0) * D + dim0);
        vok[gi] = okk;
      }
    };
    fetch_v(0);
    // partial dot products over each segment, summed across the SEG lanes
    // of a row, then key j's score moved to lane j
    float part[SEG];
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      float kf[8];
      unpack<T, 8>(kraw[i], kf);
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) d = fmaf(q8[e], kf[e], d);
#pragma unroll
      for (int off = 1; off < SEG; off <<= 1) d += __shfl_xor_sync(full, d, off);
      part[i] = d;
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const float d = __shfl_sync(full, part[i], (lane % RPI) * SEG);
      if (lane / RPI == i) dot = d;
    }
    const float s = ok ? dot * scale_log2 : -INFINITY;
    float cmax = s;
#pragma unroll
    for (int off = 16; off; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(full, cmax, off));
    if (cmax == -INFINITY) continue;  // warp-uniform: no valid key in this chunk
    const float m_new = fmaxf(m, cmax);
    const float alpha = exp2f(m - m_new);  // 0 while m is -inf
    const float p = ok ? exp2f(s - m_new) : 0.f;
    l = l * alpha + p;
#pragma unroll
    for (int i = 0; i < PD; ++i) acc[i] *= alpha;
    m = m_new;
#pragma unroll
    for (int g0 = 0; g0 < 16; g0 += G) {
      if (g0 > 0) fetch_v(g0);
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        // an invalid entry contributes exactly zero: its slice (read from
        // row 0) is replaced by zeros, whatever row 0 holds
        const float pk = __shfl_sync(full, p, 2 * (g0 + gi) + half);
        float vf[PD];
        unpack<T, PD>(vraw[gi], vf);
#pragma unroll
        for (int i = 0; i < PD; ++i) acc[i] = fmaf(pk, vok[gi] ? vf[i] : 0.f, acc[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PD; ++i) acc[i] += __shfl_xor_sync(full, acc[i], 16);
#pragma unroll
  for (int off = 16; off; off >>= 1) l += __shfl_xor_sync(full, l, off);
  if (__any_sync(full, bad) && lane == 0 && status) atomicOr(status, VGGT_STATUS_BAD_INDEX);
  if (half == 0) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint32_t w[PD / 2];
#pragma unroll
    for (int i = 0; i < PD / 2; ++i) w[i] = ElemOps<T>::pack2(acc[2 * i] * inv, acc[2 * i + 1] * inv);
    *reinterpret_cast<typename Vec<PD>::type*>(out + r * D + dim0) =
        *reinterpret_cast<const typename Vec<PD>::type*>(w);
  }
}

template <typename T>
cudaError_t launch_t(const TokenAttnArgs& a, cudaStream_t stream) {
  const unsigned grid = (unsigned)((a.n_queries + WARPS - 1) / WARPS);
  const T* q = static_cast<const T*>(a.q);
  const T* k = static_cast<const T*>(a.k);
  const T* v = static_cast<const T*>(a.v);
  T* out = static_cast<T*>(a.out);
  const float sl2 = a.scale * 1.4426950408889634f;
  switch (a.dim) {
    case 32:
      token_attn_kernel<T, 32><<<grid, WARPS * 32, 0, stream>>>(
          q, k, v, a.indices, a.index_stride, a.n_queries, a.n_keys, a.topk, sl2, out, a.status);
      break;
    case 64:
      token_attn_kernel<T, 64><<<grid, WARPS * 32, 0, stream>>>(
          q, k, v, a.indices, a.index_stride, a.n_queries, a.n_keys, a.topk, sl2, out, a.status);
      break;
    case 128:
      token_attn_kernel<T, 128><<<grid, WARPS * 32, 0, stream>>>(
          q, k, v, a.indices, a.index_stride, a.n_queries, a.n_keys, a.topk, sl2, out, a.status);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace tokattn

cudaError_t launch_token_attention(const TokenAttnArgs& a, cudaStream_t stream) {
  if (a.n_queries == 0) return cudaSuccess;
  if (a.dtype == VGGT_DTYPE_BF16) return tokattn::launch_t<__nv_bfloat16>(a, stream);
  return tokattn::launch_t<__half>(a, stream);
}

}  // namespace vggt
