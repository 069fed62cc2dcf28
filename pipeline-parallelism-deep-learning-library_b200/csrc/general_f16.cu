// general_f16.cu -- f16 contraction with the op API's rounding: one rounding to f16 of a
// double-float dot product (src/ops/contraction.rs:147-160, 829-836 route every f16 product to
// `contract_general_f16`, shaders/contraction.metal:445-702), and the K = 0 / alpha = 0 scale
// rounded once (tests/contraction_test.rs:445-470: beta = -0.999 times f16 0x0DDC is 0x8DDB, not
// the doubly rounded 0x8DDA).
//
// f16 x f16 products are exact in f32, so the only rounding inside the dot is the running sum,
// kept as an unevaluated pair hi + lo (about 48 significant bits): each product is added with
// Knuth's two-sum, the error term folded into lo.  alpha and beta * C join the pair the same way
// (Dekker's two-product, an FMA here), and the pair is rounded once to f16: round hi to the
// nearest f16 z, take the exact residual (hi - z) + lo, and step to z's neighbour when the
// residual passes half the gap to it (ties to even).  Non-finite sums fall back to IEEE
// arithmetic on hi + lo, as the reference does.  These steps are fixed by the result bits the
// reference produces, so they are the same steps; the code is this file's own.
//
// The kernel reads A, B and C in place through any strides (up to 8 axes per index group), so
// f16 operands are never staged.  One 16 x 16 block of outputs per CTA; A and B tiles of 16 along
// K go through shared memory as f32 (exact); every thread sums its output's products in k order.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "general_f16.h"
#include "internal.h"

namespace {

constexpr int kT = 16;  // output tile edge and K step

__device__ __forceinline__ void two_sum(float a, float b, float& s, float& e) {
  s = __fadd_rn(a, b);
  const float v = __fsub_rn(s, a);
  e = __fadd_rn(__fsub_rn(a, __fsub_rn(s, v)), __fsub_rn(b, v));
}

__device__ __forceinline__ void two_prod(float a, float b, float& p, float& e) {
  p = __fmul_rn(a, b);
  e = __fmaf_rn(a, b, -p);
}

__device__ __forceinline__ bool finite3(float a, float b, float c) { return isfinite(a) && isfinite(b) && isfinite(c); }

// (hi, lo) += x
__device__ __forceinline__ void dd_add(float& hi, float& lo, float x) {
  if (!finite3(hi, lo, x)) {
    hi = __fadd_rn(__fadd_rn(hi, x), lo);
    lo = 0.0f;
    return;
  }
  float s, e;
  two_sum(hi, x, s, e);
  e = __fadd_rn(e, lo);
  two_sum(s, e, hi, lo);
}

// (hi, lo) *= s
__device__ __forceinline__ void dd_scale(float& hi, float& lo, float s) {
  if (!finite3(hi, lo, s)) {
    hi = __fmaf_rn(s, hi, __fmul_rn(s, lo));
    lo = 0.0f;
    return;
  }
  float p1, e1, p2, e2;
  two_prod(s, hi, p1, e1);
  two_prod(s, lo, p2, e2);
  hi = p1;
  lo = e1;
  dd_add(hi, lo, p2);
  dd_add(hi, lo, e2);
}

// Width of the gap from the finite f16 `z` to its neighbour above (up) or below (down) in
// magnitude: one ulp, except below a normal power of two (not the smallest normal), where the
// neighbour toward zero is half an ulp away.
__device__ __forceinline__ float f16_ulp(uint16_t zb) {
  const uint32_t mag = zb & 0x7fffu;
  if (mag < 0x0400u) return __uint_as_float(0x33800000u);  // 2^-24: subnormals and the smallest normals
  return __uint_as_float((uint32_t)((int)(mag >> 10) - 25 + 127) << 23);
}

__device__ __forceinline__ uint16_t f16_step(uint16_t b, bool up) {
  const bool neg = (b & 0x8000u) != 0;
  if (up != neg) return (uint16_t)(b + 1);
  if ((b & 0x7fffu) == 0) return up ? (uint16_t)0x0001 : (uint16_t)0x8001;
  return (uint16_t)(b - 1);
}

// hi + lo rounded once to f16 (ties to even); an f16 overflow of hi is taken as is.
__device__ __forceinline__ uint16_t dd_to_f16(float hi, float lo) {
  if (!isfinite(hi) || !isfinite(lo)) return __half_as_ushort(__float2half_rn(__fadd_rn(hi, lo)));
  uint16_t z = __half_as_ushort(__float2half_rn(hi));
  if ((z & 0x7c00u) == 0x7c00u) return z;
  const float zf = __half2float(__ushort_as_half(z));
  float r, rl;
  two_sum(__fsub_rn(hi, zf), lo, r, rl);  // hi - zf is exact
  const float ulp = f16_ulp(z);
  const uint32_t e = (z >> 10) & 0x1fu;
  const bool pow2 = (z & 0x03ffu) == 0 && e >= 2;
  const float away = __fmul_rn(ulp, 0.5f), toward = pow2 ? __fmul_rn(ulp, 0.25f) : away;
  const bool neg = (z & 0x8000u) != 0;
  const float up_lim = neg ? toward : away;   // half the gap to the next f16 above
  const float dn_lim = neg ? away : toward;   // half the gap to the next f16 below
  const bool odd = (z & 1u) != 0;
  if (r > up_lim || (r == up_lim && (rl > 0.0f || (rl == 0.0f && odd)))) return f16_step(z, true);
  if (r < -dn_lim || (r == -dn_lim && (rl < 0.0f || (rl == 0.0f && odd)))) return f16_step(z, false);
  return z;
}

__device__ __forceinline__ int64_t decode(uint64_t idx, const lc::GenGroup& g, int which) {
  int64_t off = 0;
  for (int i = g.n - 1; i >= 0; i--) {
    const uint64_t q = idx / g.ext[i];
    off += (int64_t)(idx - q * g.ext[i]) * g.st[which][i];
    idx = q;
  }
  return off;
}

// alpha * (hi, lo) + beta * c, rounded once
__device__ __forceinline__ uint16_t finish_f16(float hi, float lo, float alpha, float beta, const uint16_t* cp) {
  dd_scale(hi, lo, alpha);
  if (beta != 0.0f) {
    const float c = __half2float(__ushort_as_half(*cp));
    if (!finite3(hi, lo, c)) return __half_as_ushort(__float2half_rn(__fadd_rn(__fadd_rn(hi, lo), __fmul_rn(beta, c))));
    float bh, bl;
    two_prod(beta, c, bh, bl);
    dd_add(hi, lo, bh);
    dd_add(hi, lo, bl);
  }
  return dd_to_f16(hi, lo);
}

__global__ void __launch_bounds__(kT * kT) general_f16_kernel(const __grid_constant__ lc::GenParams p) {
  __shared__ float as[kT][kT + 1];
  __shared__ float bs[kT][kT + 1];
  const int tx = threadIdx.x % kT, ty = threadIdx.x / kT;
  const uint64_t n0 = (uint64_t)blockIdx.x * kT, m0 = (uint64_t)blockIdx.y * kT;
  for (uint64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
    const int64_t ab = (int64_t)p.a_off + decode(bt, p.gb, 0);
    const int64_t bb = (int64_t)p.b_off + decode(bt, p.gb, 1);
    const int64_t cb = (int64_t)p.c_off + decode(bt, p.gb, 2);
    // this thread's loads: A row m0 + ty, B column n0 + tx
    const uint64_t lm = m0 + ty, ln = n0 + tx;
    const int64_t a_row = lm < p.m ? ab + decode(lm, p.gm, 0) : 0;
    const int64_t b_col = ln < p.n ? bb + decode(ln, p.gn, 1) : 0;
    float hi = 0.0f, lo = 0.0f;
    for (uint64_t k0 = 0; k0 < p.k; k0 += kT) {
      __syncthreads();
      const uint64_t ka = k0 + tx, kb = k0 + ty;
      as[ty][tx] = (lm < p.m && ka < p.k) ? __half2float(__ushort_as_half(p.a[a_row + decode(ka, p.gk, 0)])) : 0.0f;
      bs[ty][tx] = (ln < p.n && kb < p.k) ? __half2float(__ushort_as_half(p.b[b_col + decode(kb, p.gk, 1)])) : 0.0f;
      __syncthreads();
      const int kk_end = p.k - k0 < (uint64_t)kT ? (int)(p.k - k0) : kT;
      for (int kk = 0; kk < kk_end; kk++) dd_add(hi, lo, __fmul_rn(as[ty][kk], bs[kk][tx]));
    }
    if (lm < p.m && ln < p.n) {
      uint16_t* cp = p.c + cb + decode(lm, p.gm, 2) + decode(ln, p.gn, 2);
      *cp = finish_f16(hi, lo, p.alpha, p.beta, cp);
    }
  }
}

// C = beta * C rounded once (beta != 0), or +0 (beta == 0): the f16 Fill plan
__global__ void __launch_bounds__(256) scale_f16_kernel(const __grid_constant__ lc::GenParams p) {
  const uint64_t total = p.batch * p.m * p.n;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t col = i % p.n, rest = i / p.n, row = rest % p.m, bt = rest / p.m;
    uint16_t* cp = p.c + p.c_off + decode(bt, p.gb, 2) + decode(row, p.gm, 2) + decode(col, p.gn, 2);
    if (p.beta == 0.0f) {  // C is not read: a NaN in it cannot survive
      *cp = 0;
      continue;
    }
    // the exact product beta * c, rounded once; IEEE arithmetic when anything is not finite
    const float c = __half2float(__ushort_as_half(*cp));
    float hi = 0.0f, lo = 0.0f;
    if (isfinite(p.beta) && isfinite(c)) two_prod(p.beta, c, hi, lo);
    if (!isfinite(p.beta) || !isfinite(c) || !isfinite(hi) || !isfinite(lo))
      *cp = __half_as_ushort(__float2half_rn(__fmul_rn(p.beta, c)));
    else
      *cp = dd_to_f16(hi, lo);
  }
}

}  // namespace

namespace lc {

lc_status general_f16_run(lc_context* ctx, cudaStream_t s, const GenParams& p, bool fill) {
  if (p.m == 0 || p.n == 0 || p.batch == 0) return LC_OK;
  if (fill) {
    const uint64_t total = p.batch * p.m * p.n;
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((total + 255) / 256, (uint64_t)ctx->sm_count * 8));
    scale_f16_kernel<<<grid, 256, 0, s>>>(p);
    record_launch(ctx, p.beta == 0.0f ? "contract_zero_f16" : "contract_scale_f16");
  } else {
    const uint64_t gx = (p.n + kT - 1) / kT, gy = (p.m + kT - 1) / kT;
    if (gx > 0x7fffffffull || gy > 65535) return fail(LC_ERR_INVALID_ARGUMENT, "f16 contraction output too large");
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)std::min<uint64_t>(p.batch, 65535));
    general_f16_kernel<<<grid, kT * kT, 0, s>>>(p);
    record_launch(ctx, "contract_general_f16");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "f16 contraction launch");
  return LC_OK;
}

}  // namespace lc
