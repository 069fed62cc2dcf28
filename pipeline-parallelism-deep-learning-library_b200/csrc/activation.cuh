// activation.cuh -- the GELU of the reference's CPU backend, shared by the standalone training
// ops (elementwise.cu) and the GEMM's fused epilogues (gemm_tc.cu), so that both give the same
// bits.  f32 throughout, every operation rounded on its own (the library builds with
// --fmad=false).
#pragma once
#include <cuda_runtime.h>

namespace lcd {

// GELU with the reference's Abramowitz-Stegun 7.1.26 erf, in f32 (crates/cpu/src/lib.rs:809-853).
__device__ __forceinline__ float erf_as(float x) {
  const float A1 = 0.254829592f, A2 = 0.284496736f, A3 = 1.421413741f, A4 = 1.453152027f, A5 = 1.061405429f;
  float sign = signbit(x) ? -1.0f : 1.0f;
  x = fabsf(x);
  float t = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(0.3275911f, x)));
  float poly = __fmul_rn(A5, t);
  poly = __fmul_rn(__fsub_rn(poly, A4), t);
  poly = __fmul_rn(__fadd_rn(poly, A3), t);
  poly = __fmul_rn(__fsub_rn(poly, A2), t);
  poly = __fmul_rn(__fadd_rn(poly, A1), t);
  return __fmul_rn(sign, __fsub_rn(1.0f, __fmul_rn(poly, expf(-__fmul_rn(x, x)))));
}

__device__ __forceinline__ float gelu1(float x) {
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erf_as(__fmul_rn(x, 0.70710678118654752440f))));
}

__device__ __forceinline__ float gelu_prime1(float x) {
  float phi = __fmul_rn(0.5f, __fadd_rn(1.0f, erf_as(__fmul_rn(x, 0.70710678118654752440f))));
  float pdf = __fmul_rn(expf(__fmul_rn(__fmul_rn(-0.5f, x), x)), 0.3989422804014327f);
  return __fadd_rn(phi, __fmul_rn(x, pdf));
}

}  // namespace lcd
