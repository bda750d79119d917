// Shared device helpers for the vggt_sparse kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "vggt_sparse.h"

namespace vggt {

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------
template <typename T>
struct ElemOps;

template <>
struct ElemOps<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to_float2(uint32_t packed) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&packed);
    return __bfloat1622float2(h);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ __nv_bfloat16 from_float(float a) {
    return __float2bfloat16_rn(a);
  }
};

template <>
struct ElemOps<__half> {
  static __device__ __forceinline__ float2 to_float2(uint32_t packed) {
    __half2 h = *reinterpret_cast<__half2*>(&packed);
    return __half22float2(h);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ __half from_float(float a) { return __float2half_rn(a); }
};

// ---------------------------------------------------------------------------
// Deterministic selection arithmetic shared with the CPU oracle.
//
// The mass-threshold rule needs softmax weights whose rounding is identical on
// the GPU and in the numpy restatement, so they are computed with explicitly
// rounded fp32 multiplies/adds (no FMA contraction) and a polynomial written
// from the Taylor series of 2^f = exp(f ln 2) (coefficients (ln 2)^k / k!),
// then quantised to integers so that every later sum is exact and
// order-independent.
// ---------------------------------------------------------------------------
constexpr int kMassFracBits = 40;  // weight w in (0,1] -> floor(w * 2^40)
constexpr int kTauBits = 24;       // tau is represented as round(tau * 2^24) / 2^24

__device__ __forceinline__ float det_exp2_poly(float f) {
  // Horner over c7..c0, c_k = fp32((ln 2)^k / k!)
  float p = __uint_as_float(0x377fe5feu);
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x39218489u));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3aaec3ffu));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3c1d955bu));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3d635847u));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3e75fdf0u));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3f317218u));
  p = __fadd_rn(__fmul_rn(p, f), 1.0f);
  return p;
}

// Quantised softmax weight of a logit x = s - rowmax (x <= 0), in units of 2^-40.
__device__ __forceinline__ uint64_t det_mass_weight(float s, float rowmax) {
  float x = __fsub_rn(s, rowmax);
  float t = __fmul_rn(x, __uint_as_float(0x3fb8aa3bu));  // x * fp32(log2 e)
  if (!(t >= -64.0f)) return 0ull;                       // below 2^-64: quantises to 0
  float n = rintf(t);
  float f = __fsub_rn(t, n);  // exact
  float p = det_exp2_poly(f);
  int ni = (int)n;            // in [-64, 0]
  float scale = __uint_as_float((uint32_t)(ni + 127) << 23);  // 2^n, exact
  float w = __fmul_rn(p, scale);
  float wq = __fmul_rn(w, 1099511627776.0f);  // * 2^40, exact
  return (uint64_t)floorf(wq);
}

// Monotone uint32 key of an fp32 score: larger score -> larger key; -0 == +0.
__device__ __forceinline__ uint32_t score_key(float s) {
  s = __fadd_rn(s, 0.0f);  // canonicalise -0.0 to +0.0
  uint32_t b = __float_as_uint(s);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Mass target T = ceil(tau_num * W / 2^24) evaluated exactly in 64-bit pieces.
__device__ __forceinline__ uint64_t mass_target(uint64_t total, uint64_t tau_num) {
  uint64_t hi = total >> kTauBits;
  uint64_t lo = total & ((1ull << kTauBits) - 1ull);
  uint64_t prod_lo = tau_num * lo;  // < 2^48
  uint64_t ceil_lo = (prod_lo + ((1ull << kTauBits) - 1ull)) >> kTauBits;
  return tau_num * hi + ceil_lo;
}

// ---------------------------------------------------------------------------
// Small PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace vggt
