// elementwise.cu -- correctly rounded sqrt / reciprocal over strided views, and the Backend
// training ops (add_bias, bias_grad, mse_grad, sgd_step, convert, gelu, relu and their
// backwards).
//
// Bandwidth layout: a contiguous pair of views runs a 16-byte vector grid-stride loop sized to
// the SM count (HBM-bound: 8 bytes moved per element); any other layout runs a per-element
// mixed-radix decode over at most 8 merged axes.  All arithmetic is IEEE f32 with no flush to
// zero and no FMA contraction (the library is built with -fmad=false), one rounding per
// written operation, as crates/core/src/lib.rs:98-102 requires.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "activation.cuh"
#include "internal.h"

namespace {

struct Strided {
  int rank;
  uint64_t count;
  uint64_t src_off, dst_off;
  uint64_t shape[LC_MAX_RANK];
  uint64_t src_st[LC_MAX_RANK];
  uint64_t dst_st[LC_MAX_RANK];
};

// Merges axes that are contiguous in both views (outer stride == inner stride * inner extent).
Strided merge_pair(const lc_view& src, const lc_view& dst) {
  Strided p{};
  p.src_off = src.offset;
  p.dst_off = dst.offset;
  p.count = lc::numel(src);
  int r = 0;
  for (int d = 0; d < src.rank; d++) {
    if (src.shape[d] == 1) continue;
    if (r > 0 && p.src_st[r - 1] == src.strides[d] * src.shape[d] && p.dst_st[r - 1] == dst.strides[d] * src.shape[d]) {
      p.shape[r - 1] *= src.shape[d];
      p.src_st[r - 1] = src.strides[d];
      p.dst_st[r - 1] = dst.strides[d];
      continue;
    }
    p.shape[r] = src.shape[d];
    p.src_st[r] = src.strides[d];
    p.dst_st[r] = dst.strides[d];
    r++;
  }
  if (r == 0) {
    p.shape[0] = 1;
    p.src_st[0] = 1;
    p.dst_st[0] = 1;
    r = 1;
  }
  p.rank = r;
  return p;
}

__device__ __forceinline__ void decode(const Strided& p, uint64_t i, uint64_t* so, uint64_t* dof) {
  uint64_t s = p.src_off, d = p.dst_off;
  for (int a = p.rank - 1; a >= 0; a--) {
    uint64_t n = p.shape[a];
    uint64_t c = i % n;
    i /= n;
    s += c * p.src_st[a];
    d += c * p.dst_st[a];
  }
  *so = s;
  *dof = d;
}

// (x as f64).sqrt() as f32.  __fsqrt_rn is IEEE correctly rounded (no ftz in this build), which
// equals the double-then-round value because 53 >= 2*24 + 2.  NaN inputs keep sign and payload
// and become quiet, and a negative input gives the x86 default NaN 0xffc00000, as the Rust
// expression does on the reference's hosts.
__device__ __forceinline__ float sqrt_ref(float x) {
  uint32_t b = __float_as_uint(x);
  if ((b & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(b | 0x00400000u);
  if (x < 0.0f) return __uint_as_float(0xffc00000u);
  return __fsqrt_rn(x);
}

// (1.0 / x as f64) as f32: __frcp_rn is the correctly rounded reciprocal (subnormal inputs and
// results kept).  NaN keeps sign and payload and becomes quiet.
__device__ __forceinline__ float rcp_ref(float x) {
  uint32_t b = __float_as_uint(x);
  if ((b & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(b | 0x00400000u);
  return __frcp_rn(x);
}

template <int OP>
__device__ __forceinline__ float apply(float x) {
  if constexpr (OP == 0) return sqrt_ref(x);
  else return rcp_ref(x);
}

template <int OP>
__global__ void __launch_bounds__(256) unary_vec_kernel(const float4* __restrict__ src, float4* __restrict__ dst,
                                                         uint64_t n4) {
  uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  // Four independent 16-byte loads in flight per thread before the first store.
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; u++) {
      float4 r = make_float4(apply<OP>(v[u].x), apply<OP>(v[u].y), apply<OP>(v[u].z), apply<OP>(v[u].w));
      __stcs(dst + i + u * stride, r);
    }
  }
  for (; i < n4; i += stride) {
    float4 v = __ldcs(src + i);
    __stcs(dst + i, make_float4(apply<OP>(v.x), apply<OP>(v.y), apply<OP>(v.z), apply<OP>(v.w)));
  }
}

template <int OP>
__global__ void unary_scalar_kernel(const float* __restrict__ src, float* __restrict__ dst, uint64_t n) {
  uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i < n) dst[i] = apply<OP>(src[i]);
}

template <int OP>
__global__ void unary_strided_kernel(const float* src, float* dst, Strided p) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < p.count; i += stride) {
    uint64_t so, dof;
    decode(p, i, &so, &dof);
    dst[dof] = apply<OP>(src[so]);
  }
}

// ---- complex reciprocal (src/ops/reciprocal.rs:17-31, shaders/reciprocal.metal:141-330) -------
// Smith's algorithm on split floats: a nonzero finite value is a significand m with |m| in
// [1, 2) and an exponent e, x = m * 2^e, so no intermediate overflows, underflows or becomes
// subnormal.  Each product or sum of significands is one IEEE f32 rounding, each division is
// the dividend times the correctly rounded reciprocal of the divisor, and the parts are packed
// into f32 once (a subnormal part rounds the 24-bit significand right, nearest even).  The
// specials follow C99 Annex G as the reference documents them.
struct Split {
  float m;
  int e;
};

// a nonzero finite f32 (subnormals normalised)
__device__ __forceinline__ Split split_of(uint32_t b) {
  const uint32_t ex = (b >> 23) & 0xffu, fr = b & 0x007fffffu, sg = b & 0x80000000u;
  if (ex == 0u) {
    const int sh = __clz((int)fr) - 8;
    return {__uint_as_float(((fr << sh) & 0x007fffffu) | (127u << 23) | sg), -126 - sh};
  }
  return {__uint_as_float((b & 0x807fffffu) | (127u << 23)), (int)ex - 127};
}

__device__ __forceinline__ Split split_mul(Split a, Split b) {
  if (a.m == 0.0f || b.m == 0.0f) return {__fmul_rn(a.m, b.m), 0};
  const float p = __fmul_rn(a.m, b.m);
  return fabsf(p) >= 2.0f ? Split{p * 0.5f, a.e + b.e + 1} : Split{p, a.e + b.e};
}

__device__ __forceinline__ Split split_rcp(Split a) {
  const float inv = __frcp_rn(a.m);
  return fabsf(inv) < 1.0f ? Split{inv * 2.0f, -a.e - 1} : Split{inv, -a.e};
}

// a + b for parts of one sign (Smith's denominator never cancels); b shifted by the exponent
// gap, dropped from 25 binades down
__device__ __forceinline__ Split split_add(Split a, Split b) {
  if (b.m == 0.0f) return a;
  if (a.m == 0.0f) return b;
  if (a.e < b.e) {
    const Split t = a;
    a = b;
    b = t;
  }
  const int gap = a.e - b.e;
  if (gap >= 25) return a;
  const float s = __fadd_rn(a.m, __fmul_rn(b.m, __uint_as_float((uint32_t)(127 - gap) << 23)));
  return fabsf(s) >= 2.0f ? Split{s * 0.5f, a.e + 1} : Split{s, a.e};
}

__device__ __forceinline__ bool split_abs_ge(Split a, Split b) {
  const bool az = a.m == 0.0f, bz = b.m == 0.0f;
  if (az) return bz;
  if (bz) return true;
  if (a.e != b.e) return a.e > b.e;
  return fabsf(a.m) >= fabsf(b.m);
}

__device__ __forceinline__ uint32_t split_bits(Split s) {
  const uint32_t raw = __float_as_uint(s.m), sign = raw & 0x80000000u;
  if ((raw & 0x7fffffffu) == 0u) return sign;
  if (s.e >= 128) return sign | 0x7f800000u;
  if (s.e >= -126) return (raw & 0x807fffffu) | ((uint32_t)(s.e + 127) << 23);
  const uint32_t sh = (uint32_t)(-s.e - 126);
  if (sh >= 25u) return sign;
  const uint32_t mant = (raw & 0x007fffffu) | 0x00800000u;
  const uint32_t kept = mant >> sh, rem = mant & ((1u << sh) - 1u), half = 1u << (sh - 1u);
  // at most 2^23: a subnormal, or the carry into the smallest normal, which has these bits
  return sign | ((rem > half || (rem == half && (kept & 1u))) ? kept + 1u : kept);
}

__device__ __forceinline__ uint2 rcp_c32(uint2 z) {
  const uint32_t ab = z.x, bb = z.y;
  const bool a_top = ((ab >> 23) & 0xffu) == 0xffu, b_top = ((bb >> 23) & 0xffu) == 0xffu;
  const bool a_inf = a_top && !(ab & 0x007fffffu), b_inf = b_top && !(bb & 0x007fffffu);
  if (a_inf || b_inf) return make_uint2(ab & 0x80000000u, ~bb & 0x80000000u);
  if (a_top || b_top) return make_uint2(0x7fc00000u, 0x7fc00000u);  // a NaN part
  if (!(bb & 0x7fffffffu)) return make_uint2(__float_as_uint(__frcp_rn(__uint_as_float(ab))), ~bb & 0x80000000u);
  if (!(ab & 0x7fffffffu)) return make_uint2(ab & 0x80000000u, __float_as_uint(__frcp_rn(__uint_as_float(bb))) ^ 0x80000000u);
  const Split a = split_of(ab), b = split_of(bb);
  if (split_abs_ge(a, b)) {
    const Split r = split_mul(b, split_rcp(a));                  // b / a
    const Split inv = split_rcp(split_add(a, split_mul(b, r)));  // 1 / (a + b r)
    return make_uint2(split_bits(inv), split_bits(split_mul(Split{-r.m, r.e}, inv)));
  }
  const Split r = split_mul(a, split_rcp(b));                    // a / b
  const Split inv = split_rcp(split_add(b, split_mul(a, r)));    // 1 / (a r + b)
  return make_uint2(split_bits(split_mul(r, inv)), split_bits(Split{-inv.m, inv.e}));
}

// One 16-byte vector (two complex values) per thread per pass.  (Four vectors in flight per
// thread measured slower: the branchy special-case paths keep the compiler from interleaving
// the values' dependent chains, and the extra registers cost occupancy.)
__global__ void __launch_bounds__(256) rcp_c32_vec_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                          uint64_t n2) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n2; i += stride) {
    const uint4 v = __ldcs(src + i);
    const uint2 lo = rcp_c32(make_uint2(v.x, v.y)), hi = rcp_c32(make_uint2(v.z, v.w));
    __stcs(dst + i, make_uint4(lo.x, lo.y, hi.x, hi.y));
  }
}

__global__ void rcp_c32_scalar_kernel(const uint2* __restrict__ src, uint2* __restrict__ dst, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) dst[i] = rcp_c32(src[i]);
}

__global__ void rcp_c32_strided_kernel(const uint2* src, uint2* dst, Strided p) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < p.count; i += stride) {
    uint64_t so, dof;
    decode(p, i, &so, &dof);
    dst[dof] = rcp_c32(src[so]);
  }
}

unsigned grid_for(lc_context* ctx, uint64_t work, unsigned block) {
  uint64_t want = (work + block - 1) / block;
  uint64_t cap = (uint64_t)ctx->sm_count * 32;  // 32 blocks per SM: 6.33 TB/s on sqrt, 5.72 at 8
  if (want > cap) want = cap;
  if (want == 0) want = 1;
  return (unsigned)want;
}

template <int OP>
lc_status run_unary(lc_context* ctx, void* stream, const lc_view* srcp, const lc_view* dstp, const char* opname) {
  using namespace lc;
  if (ctx == nullptr || srcp == nullptr || dstp == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  const lc_view& src = *srcp;
  const lc_view& dst = *dstp;
  // src/ops/sqrt.rs:121-167 `prepare` order: validate, dtype, shape, rank, overlap, empty,
  // injective destination.
  lc_status st = validate(src, "src");
  if (st) return st;
  if ((st = validate(dst, "dst"))) return st;
  // sqrt: real f32; reciprocal: real f32 or complex [f32; 2] (src/ops/reciprocal.rs:49-61)
  const bool complex = OP == 1 && src.dtype == LC_C32 && dst.dtype == LC_C32;
  if (!complex && (src.dtype != LC_F32 || dst.dtype != LC_F32))
    return fail(LC_ERR_INVALID_ARGUMENT, std::string(opname) + (OP == 1 ? " supports f32 and complex f32 views"
                                                                        : " supports real f32 views"));
  if (src.rank != dst.rank || memcmp(src.shape, dst.shape, sizeof(uint64_t) * src.rank) != 0)
    return fail(LC_ERR_INVALID_ARGUMENT, std::string(opname) + " shape mismatch");
  bool inplace = same_view(src, dst);
  if (!inplace && may_overlap(src, dst))
    return fail(LC_ERR_OVERLAP, std::string(opname) +
                                    " views overlap; in-place requires the same buffer, offset, shape, and strides");
  if (is_empty(src)) return LC_OK;
  if (!is_injective(dst))
    return fail(LC_ERR_INVALID_ARGUMENT, std::string(opname) + " destination is not injective; parallel stores would alias");
  cudaStream_t s = stream_of(ctx, stream);
  uint64_t n = numel(src);
  if (complex) {
    const uint2* zp = static_cast<const uint2*>(src.data) + src.offset;
    uint2* wp = static_cast<uint2*>(dst.data) + dst.offset;
    if (is_contiguous(src) && is_contiguous(dst)) {
      const bool aligned = (reinterpret_cast<uintptr_t>(zp) % 16 == 0) && (reinterpret_cast<uintptr_t>(wp) % 16 == 0);
      const uint64_t n2 = aligned ? n / 2 : 0;
      if (n2) {
        rcp_c32_vec_kernel<<<grid_for(ctx, n2, 256), 256, 0, s>>>(reinterpret_cast<const uint4*>(zp),
                                                                  reinterpret_cast<uint4*>(wp), n2);
        record_launch(ctx, "reciprocal_c32_vec");
      }
      if (n - 2 * n2) {
        rcp_c32_scalar_kernel<<<grid_for(ctx, n - 2 * n2, 256), 256, 0, s>>>(zp + 2 * n2, wp + 2 * n2, n - 2 * n2);
        record_launch(ctx, "reciprocal_c32_scalar");
      }
    } else {
      Strided p = merge_pair(src, dst);
      rcp_c32_strided_kernel<<<grid_for(ctx, n, 256), 256, 0, s>>>(static_cast<const uint2*>(src.data),
                                                                   static_cast<uint2*>(dst.data), p);
      record_launch(ctx, "reciprocal_c32_strided");
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, opname);
    return LC_OK;
  }
  const float* sp = static_cast<const float*>(src.data) + src.offset;
  float* dp = static_cast<float*>(dst.data) + dst.offset;
  if (is_contiguous(src) && is_contiguous(dst)) {
    bool aligned = (reinterpret_cast<uintptr_t>(sp) % 16 == 0) && (reinterpret_cast<uintptr_t>(dp) % 16 == 0);
    if (aligned && n >= 4) {
      uint64_t n4 = n / 4;
      unary_vec_kernel<OP><<<grid_for(ctx, n4, 256) * 1, 256, 0, s>>>(reinterpret_cast<const float4*>(sp),
                                                                       reinterpret_cast<float4*>(dp), n4);
      record_launch(ctx, OP == 0 ? "sqrt_vec" : "reciprocal_vec");
      uint64_t tail = n - n4 * 4;
      if (tail) {
        unary_scalar_kernel<OP><<<1, 32, 0, s>>>(sp + n4 * 4, dp + n4 * 4, tail);
        record_launch(ctx, OP == 0 ? "sqrt_tail" : "reciprocal_tail");
      }
    } else {
      unary_scalar_kernel<OP><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(sp, dp, n);
      record_launch(ctx, OP == 0 ? "sqrt_scalar" : "reciprocal_scalar");
    }
  } else {
    Strided p = merge_pair(src, dst);
    unary_strided_kernel<OP><<<grid_for(ctx, n, 256), 256, 0, s>>>(static_cast<const float*>(src.data),
                                                                  static_cast<float*>(dst.data), p);
    record_launch(ctx, OP == 0 ? "sqrt_strided" : "reciprocal_strided");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, opname);
  return LC_OK;
}

// ---------------------------------------------------------------------------------------------
// Backend training ops (crates/cuda/train.cu semantics, crates/cpu/src/lib.rs:372-533 math).
// ---------------------------------------------------------------------------------------------

__global__ void add_bias_kernel(const float* x, const float* b, float* y, uint64_t rows, uint64_t cols) {
  const uint64_t n = rows * cols, stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = __fadd_rn(x[i], b[i % cols]);
}

// Column sums in row order (the reference's order), one thread per column, then db += s.
__global__ void bias_grad_kernel(const float* dpre, float* db, uint64_t rows, uint64_t cols) {
  uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.0f;
  for (uint64_t r = 0; r < rows; r++) s = __fadd_rn(s, dpre[r * cols + c]);
  db[c] = __fadd_rn(db[c], s);
}

// mse_grad stage 1: dy = (2*d)/n exactly as the reference (bitwise), and per-block partial sums
// of d*d in a fixed tree order (deterministic; the order differs from the reference's
// sequential sum, so the loss matches within rounding).
constexpr int kMseBlock = 512;
__global__ void __launch_bounds__(kMseBlock) mse_stage1(const float* y, const float* t, float* dy, uint64_t n, float nf,
                                                         float* partials) {
  __shared__ float red[kMseBlock];
  float acc = 0.0f;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float d = __fsub_rn(y[i], t[i]);
    acc = __fadd_rn(acc, __fmul_rn(d, d));
    dy[i] = __fdiv_rn(__fmul_rn(2.0f, d), nf);
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = kMseBlock / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) partials[blockIdx.x] = red[0];
}

__global__ void __launch_bounds__(kMseBlock) mse_stage2(const float* partials, int count, float nf, float* loss) {
  __shared__ float red[kMseBlock];
  float acc = 0.0f;
  for (int i = threadIdx.x; i < count; i += kMseBlock) acc = __fadd_rn(acc, partials[i]);
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = kMseBlock / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = __fdiv_rn(red[0], nf);
}

__global__ void sgd_kernel(float* w, float* dw, uint64_t n, float lr) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float step = __fmul_rn(lr, dw[i]);
    w[i] = __fsub_rn(w[i], step);
    dw[i] = 0.0f;
  }
}

// crates/cpu/src/lib.rs:725-731 f32_bits_to_bf16.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  uint32_t bits = __float_as_uint(x);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
  uint32_t lsb = (bits >> 16) & 1u;
  return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}

__global__ void convert_f32_bf16_kernel(const float* x, uint16_t* y, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) y[i] = f32_to_bf16_bits(x[i]);
}

__global__ void convert_bf16_f32_kernel(const uint16_t* x, float* y, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = __uint_as_float(((uint32_t)x[i]) << 16);
}

using lcd::erf_as;
using lcd::gelu1;
using lcd::gelu_prime1;

template <int OP>  // 0 gelu, 1 relu
__global__ void act_kernel(const float* x, float* y, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float v = x[i];
    y[i] = OP == 0 ? gelu1(v) : (v > 0.0f ? v : 0.0f);
  }
}

template <int OP>
__global__ void act_backward_kernel(const float* pre, const float* dy, float* dx, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float p = pre[i];
    dx[i] = OP == 0 ? __fmul_rn(dy[i], gelu_prime1(p)) : (p > 0.0f ? dy[i] : 0.0f);
  }
}

// ---- shared checks in the order Shape, Dtype, Alias, UnsupportedLayout ----------------------

bool shape_eq(const lc_view& a, const lc_view& b) {
  return a.rank == b.rank && memcmp(a.shape, b.shape, sizeof(uint64_t) * a.rank) == 0;
}

lc_status check_training(std::initializer_list<const lc_view*> all) {
  using namespace lc;
  for (const lc_view* v : all) {
    if (!packed_layout(*v)) return fail(LC_ERR_UNSUPPORTED_LAYOUT, "operand is not row-major contiguous at offset 0");
    uint64_t need = numel(*v) * dtype_size(v->dtype);
    if (need > v->buffer_bytes) return fail(LC_ERR_SHAPE, "buffer is shorter than the tensor");
  }
  return LC_OK;
}

lc_status launched(lc_context* ctx, const char* name) {
  lc::record_launch(ctx, name);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return lc::cuda_fail(e, name);
  return LC_OK;
}

}  // namespace

using namespace lc;

extern "C" {

lc_status lc_encode_sqrt(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst) {
  return run_unary<0>(ctx, stream, src, dst, "sqrt");
}

lc_status lc_sqrt(lc_context* ctx, const lc_view* src, const lc_view* dst) {
  lc_status st = lc_encode_sqrt(ctx, nullptr, src, dst);
  return st ? st : lc_sync(ctx, nullptr);
}

lc_status lc_encode_reciprocal(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst) {
  return run_unary<1>(ctx, stream, src, dst, "reciprocal");
}

lc_status lc_reciprocal(lc_context* ctx, const lc_view* src, const lc_view* dst) {
  lc_status st = lc_encode_reciprocal(ctx, nullptr, src, dst);
  return st ? st : lc_sync(ctx, nullptr);
}

lc_status lc_add_bias(lc_context* ctx, void* stream, const lc_view* x, const lc_view* b, const lc_view* y) {
  if (!ctx || !x || !b || !y) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (x->rank != 2 || !shape_eq(*x, *y) || b->rank != 1 || b->shape[0] != x->shape[1])
    return fail(LC_ERR_SHAPE, "add_bias: x [B,N], b [N], y [B,N]");
  if (x->dtype != LC_F32 || b->dtype != LC_F32 || y->dtype != LC_F32) return fail(LC_ERR_DTYPE, "add_bias: f32 only");
  if (b->data == x->data || b->data == y->data) return fail(LC_ERR_ALIAS, "add_bias: b shares storage");
  lc_status st = check_training({x, b, y});
  if (st) return st;
  uint64_t n = numel(*x);
  cudaStream_t s = stream_of(ctx, stream);
  add_bias_kernel<<<grid_for(ctx, n, 256), 256, 0, s>>>((const float*)x->data, (const float*)b->data, (float*)y->data,
                                                        x->shape[0], x->shape[1]);
  return launched(ctx, "add_bias");
}

lc_status lc_bias_grad(lc_context* ctx, void* stream, const lc_view* dpre, const lc_view* db) {
  if (!ctx || !dpre || !db) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (dpre->rank != 2 || db->rank != 1 || db->shape[0] != dpre->shape[1])
    return fail(LC_ERR_SHAPE, "bias_grad: dpre [B,N], db [N]");
  if (dpre->dtype != LC_F32 || db->dtype != LC_F32) return fail(LC_ERR_DTYPE, "bias_grad: f32 only");
  if (dpre->data == db->data) return fail(LC_ERR_ALIAS, "bias_grad: db shares storage with dpre");
  lc_status st = check_training({dpre, db});
  if (st) return st;
  if (dpre->shape[0] == 0 || dpre->shape[1] == 0) {
    record_launch(ctx, "bias_grad");
    return LC_OK;
  }
  uint64_t cols = dpre->shape[1];
  bias_grad_kernel<<<(unsigned)((cols + 255) / 256), 256, 0, stream_of(ctx, stream)>>>(
      (const float*)dpre->data, (float*)db->data, dpre->shape[0], cols);
  return launched(ctx, "bias_grad");
}

lc_status lc_mse_grad(lc_context* ctx, void* stream, const lc_view* y, const lc_view* target, const lc_view* dy,
                      float* loss) {
  if (!ctx || !y || !target || !dy || !loss) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (!shape_eq(*y, *target) || !shape_eq(*y, *dy)) return fail(LC_ERR_SHAPE, "mse_grad: shapes differ");
  uint64_t n = numel(*y);
  if (n == 0) return fail(LC_ERR_SHAPE, "mse_grad: empty tensor");
  if (y->dtype != LC_F32 || target->dtype != LC_F32 || dy->dtype != LC_F32) return fail(LC_ERR_DTYPE, "mse_grad: f32 only");
  if (dy->data == target->data) return fail(LC_ERR_ALIAS, "mse_grad: dy shares storage with target");
  lc_status st = check_training({y, target, dy});
  if (st) return st;
  cudaStream_t s = stream_of(ctx, stream);
  int blocks = (int)grid_for(ctx, n, kMseBlock);
  float* scratch = nullptr;
  if ((st = scratch_alloc(ctx, s, sizeof(float) * (blocks + 1), (void**)&scratch))) return st;
  float nf = (float)n;
  mse_stage1<<<blocks, kMseBlock, 0, s>>>((const float*)y->data, (const float*)target->data, (float*)dy->data, n, nf,
                                          scratch + 1);
  if ((st = launched(ctx, "mse_grad_partial"))) return st;
  mse_stage2<<<1, kMseBlock, 0, s>>>(scratch + 1, blocks, nf, scratch);
  if ((st = launched(ctx, "mse_grad_final"))) return st;
  float h = 0.0f;
  cudaError_t e = cudaMemcpyAsync(&h, scratch, sizeof(float), cudaMemcpyDeviceToHost, s);
  scratch_free(scratch, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "mse_grad loss readback");
  *loss = h;
  return LC_OK;
}

lc_status lc_sgd_step(lc_context* ctx, void* stream, const lc_view* w, const lc_view* dw, float lr) {
  if (!ctx || !w || !dw) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (!shape_eq(*w, *dw)) return fail(LC_ERR_SHAPE, "sgd_step: shapes differ");
  if (w->dtype != LC_F32 || dw->dtype != LC_F32) return fail(LC_ERR_DTYPE, "sgd_step: f32 only");
  if (w->data == dw->data) return fail(LC_ERR_ALIAS, "sgd_step: w and dw share storage");
  lc_status st = check_training({w, dw});
  if (st) return st;
  uint64_t n = numel(*w);
  sgd_kernel<<<grid_for(ctx, n, 256), 256, 0, stream_of(ctx, stream)>>>((float*)w->data, (float*)dw->data, n, lr);
  return launched(ctx, "sgd_step");
}

lc_status lc_convert(lc_context* ctx, void* stream, const lc_view* x, const lc_view* y) {
  if (!ctx || !x || !y) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (!shape_eq(*x, *y)) return fail(LC_ERR_SHAPE, "convert: shapes differ");
  bool f2b = x->dtype == LC_F32 && y->dtype == LC_BF16;
  bool b2f = x->dtype == LC_BF16 && y->dtype == LC_F32;
  if (!f2b && !b2f) return fail(LC_ERR_DTYPE, "convert: (f32, bf16) or (bf16, f32)");
  if (x->data == y->data) return fail(LC_ERR_ALIAS, "convert: x and y share storage");
  lc_status st = check_training({x, y});
  if (st) return st;
  uint64_t n = numel(*x);
  cudaStream_t s = stream_of(ctx, stream);
  if (f2b) {
    convert_f32_bf16_kernel<<<grid_for(ctx, n, 256), 256, 0, s>>>((const float*)x->data, (uint16_t*)y->data, n);
    return launched(ctx, "convert_f32_bf16");
  }
  convert_bf16_f32_kernel<<<grid_for(ctx, n, 256), 256, 0, s>>>((const uint16_t*)x->data, (float*)y->data, n);
  return launched(ctx, "convert_bf16_f32");
}

static lc_status unary_training(lc_context* ctx, void* stream, const lc_view* x, const lc_view* y, int op) {
  if (!ctx || !x || !y) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (x->dtype != LC_F32 || y->dtype != LC_F32) return fail(LC_ERR_DTYPE, "f32 only");
  if (!shape_eq(*x, *y)) return fail(LC_ERR_SHAPE, "shapes differ");
  lc_status st = check_training({x, y});
  if (st) return st;
  uint64_t n = numel(*x);
  cudaStream_t s = stream_of(ctx, stream);
  if (op == 0) act_kernel<0><<<grid_for(ctx, n, 256), 256, 0, s>>>((const float*)x->data, (float*)y->data, n);
  else act_kernel<1><<<grid_for(ctx, n, 256), 256, 0, s>>>((const float*)x->data, (float*)y->data, n);
  return launched(ctx, op == 0 ? "gelu" : "relu");
}

static lc_status backward_training(lc_context* ctx, void* stream, const lc_view* pre, const lc_view* dy,
                                   const lc_view* dx, int op) {
  if (!ctx || !pre || !dy || !dx) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (pre->dtype != LC_F32 || dy->dtype != LC_F32 || dx->dtype != LC_F32) return fail(LC_ERR_DTYPE, "f32 only");
  if (!shape_eq(*pre, *dy) || !shape_eq(*pre, *dx)) return fail(LC_ERR_SHAPE, "shapes differ");
  lc_status st = check_training({pre, dy, dx});
  if (st) return st;
  uint64_t n = numel(*pre);
  cudaStream_t s = stream_of(ctx, stream);
  if (op == 0)
    act_backward_kernel<0><<<grid_for(ctx, n, 256), 256, 0, s>>>((const float*)pre->data, (const float*)dy->data,
                                                                (float*)dx->data, n);
  else
    act_backward_kernel<1><<<grid_for(ctx, n, 256), 256, 0, s>>>((const float*)pre->data, (const float*)dy->data,
                                                                (float*)dx->data, n);
  return launched(ctx, op == 0 ? "gelu_backward" : "relu_backward");
}

lc_status lc_gelu(lc_context* ctx, void* stream, const lc_view* x, const lc_view* y) {
  return unary_training(ctx, stream, x, y, 0);
}
lc_status lc_relu(lc_context* ctx, void* stream, const lc_view* x, const lc_view* y) {
  return unary_training(ctx, stream, x, y, 1);
}
lc_status lc_gelu_backward(lc_context* ctx, void* stream, const lc_view* pre, const lc_view* dy, const lc_view* dx) {
  return backward_training(ctx, stream, pre, dy, dx, 0);
}
lc_status lc_relu_backward(lc_context* ctx, void* stream, const lc_view* pre, const lc_view* dy, const lc_view* dx) {
  return backward_training(ctx, stream, pre, dy, dx, 1);
}

}  // extern "C"
