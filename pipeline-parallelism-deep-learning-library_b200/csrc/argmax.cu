// argmax.cu -- index of the largest |x| (src/ops/argmax.rs, shaders/argmax.metal).
//
// Order (identical at every level of the reduction, so results are deterministic and need no
// atomics): a NaN magnitude outranks every number, a larger magnitude wins, equal magnitudes go
// to the lower index.  Magnitudes compare as integer keys: the bits of |x| (a non-negative float
// orders like its bit pattern) with every NaN mapped to 0x7fc00000, above +inf.  A candidate is
// the u64 (key << 32) | (0xffffffff - index); the larger candidate is the better one and 0 is
// the neutral element.
//
// Rank-1 (the reference op): n <= 4096 runs one block; longer inputs run up to 1024 partial
// blocks into a scratch array of candidates and one final block.
// Batched (this build's extension for the benchmark's "argmax over the last axis"): groups of
// LPR lanes own one row each (LPR = 16 for 64-float rows, 16-byte loads), shuffle-reduce, and
// write the u32 index.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <type_traits>

#include "internal.h"

namespace {

constexpr uint32_t kNanKey = 0x7fc00000u;
constexpr int kThreads = 256;
constexpr uint64_t kSinglePassMax = 4096;
constexpr uint64_t kMaxGroups = 1024;
constexpr uint64_t kItemsPerThread = 4;

__device__ __forceinline__ uint32_t key_of_bits(uint32_t bits) {
  bits &= 0x7fffffffu;
  return bits > 0x7f800000u ? kNanKey : bits;
}

__device__ __forceinline__ uint64_t cand(uint32_t key, uint64_t idx) {
  return ((uint64_t)key << 32) | (uint64_t)(0xffffffffu - (uint32_t)idx);
}

// complex magnitude keys (tests/argmax_test.rs:52-71 `mag32`), IEEE f32 with no flush
template <int MAG>
__device__ __forceinline__ uint32_t complex_key(float re, float im) {
  re = fabsf(re);
  im = fabsf(im);
  if (isnan(re) || isnan(im)) return kNanKey;
  float m;
  if (MAG == 0) {
    m = __fadd_rn(re, im);
  } else {
    float hi = fmaxf(re, im), lo = fminf(re, im);
    if (hi == 0.0f) m = 0.0f;
    else if (isinf(hi)) m = __int_as_float(0x7f800000);
    else {
      float r = __fdiv_rn(lo, hi);
      m = __fmul_rn(hi, __fsqrt_rn(__fmaf_rn(r, r, 1.0f)));
    }
  }
  return key_of_bits(__float_as_uint(m));
}

__device__ __forceinline__ uint64_t block_max(uint64_t v) {
  __shared__ uint64_t red[kThreads / 32];
  for (int o = 16; o > 0; o >>= 1) {
    uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0;
    for (int o = 16; o > 0; o >>= 1) {
      uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
      v = w > v ? w : v;
    }
  }
  return v;
}

// kind: 0 real f32, 1 complex L1, 2 complex Hypot.  Each block folds a contiguous chunk of
// indices; `out_idx` (single pass) or `partials[blockIdx.x]` receives the result.
template <int KIND>
__global__ void __launch_bounds__(kThreads) argmax_pass1(const float* x, uint64_t offset, uint64_t stride, uint64_t n,
                                                          uint64_t chunk, uint64_t* partials, uint32_t* out_idx) {
  const uint64_t begin = (uint64_t)blockIdx.x * chunk;
  const uint64_t end = min(n, begin + chunk);
  uint64_t best = 0;
  for (uint64_t i = begin + threadIdx.x; i < end; i += kThreads) {
    uint32_t key;
    if (KIND == 0) {
      key = key_of_bits(__float_as_uint(x[offset + i * stride]));
    } else {
      const float* z = x + 2 * (offset + i * stride);
      key = complex_key<KIND - 1>(z[0], z[1]);
    }
    uint64_t c = cand(key, i);
    best = c > best ? c : best;
  }
  best = block_max(best);
  if (threadIdx.x == 0) {
    if (out_idx) *out_idx = 0xffffffffu - (uint32_t)best;
    else partials[blockIdx.x] = best;
  }
}

__global__ void __launch_bounds__(kThreads) argmax_final(const uint64_t* partials, int count, uint32_t* out_idx) {
  uint64_t best = 0;
  for (int i = threadIdx.x; i < count; i += kThreads) best = partials[i] > best ? partials[i] : best;
  best = block_max(best);
  if (threadIdx.x == 0) *out_idx = 0xffffffffu - (uint32_t)best;
}

struct RowGeom {
  uint64_t rows, cols;
  uint64_t col_stride;
  int rank;  // leading axes
  uint64_t shape[LC_MAX_RANK];
  uint64_t xs[LC_MAX_RANK];
  uint64_t os[LC_MAX_RANK];
  uint64_t x_off, o_off;
  int vec;  // rows are 16-byte aligned runs of cols (multiple of 4) with unit column stride
};

__device__ __forceinline__ void row_offsets(const RowGeom& g, uint64_t r, uint64_t* xo, uint64_t* oo) {
  if (g.rank == 1) {  // leading axes collapsed to one row stride on the host: no division
    *xo = g.x_off + r * g.xs[0];
    *oo = g.o_off + r * g.os[0];
    return;
  }
  uint64_t a = g.x_off, b = g.o_off;
  for (int d = g.rank - 1; d >= 0; d--) {
    uint64_t n = g.shape[d];
    uint64_t c = r % n;
    r /= n;
    a += c * g.xs[d];
    b += c * g.os[d];
  }
  *xo = a;
  *oo = b;
}

// LPR lanes per row; rows strided over the grid.
__global__ void __launch_bounds__(kThreads) argmax_rows_kernel(const float* __restrict__ x, uint32_t* __restrict__ out,
                                                                RowGeom g, int lpr) {
  const uint64_t lane_in_row = threadIdx.x % lpr;
  const uint64_t rows_per_block = kThreads / lpr;
  const uint64_t row_stride = (uint64_t)gridDim.x * rows_per_block;
  const unsigned group_mask = lpr == 32 ? 0xffffffffu : (((1u << lpr) - 1u) << ((threadIdx.x & 31) / lpr * lpr));
  if (g.vec && g.cols == 4 * (uint64_t)lpr) {
    // one float4 per lane per row (64-float rows): load 4 rows before reducing any, so each
    // thread keeps 4 loads in flight instead of 1
    constexpr int R = 4;
    for (uint64_t r0 = (uint64_t)blockIdx.x * rows_per_block * R; r0 < g.rows; r0 += row_stride * R) {
      float4 q[R];
      uint64_t oo[R];
      bool act[R];
#pragma unroll
      for (int k = 0; k < R; k++) {
        const uint64_t r = r0 + k * rows_per_block + threadIdx.x / lpr;
        act[k] = r < g.rows;
        uint64_t xo = 0;
        oo[k] = 0;
        if (act[k]) {
          row_offsets(g, r, &xo, &oo[k]);
          q[k] = __ldcs(reinterpret_cast<const float4*>(x + xo) + lane_in_row);
        }
      }
#pragma unroll
      for (int k = 0; k < R; k++) {
        uint64_t best = 0;
        if (act[k]) {
          const uint64_t i = lane_in_row * 4;
          uint64_t c0 = cand(key_of_bits(__float_as_uint(q[k].x)), i);
          uint64_t c1 = cand(key_of_bits(__float_as_uint(q[k].y)), i + 1);
          uint64_t c2 = cand(key_of_bits(__float_as_uint(q[k].z)), i + 2);
          uint64_t c3 = cand(key_of_bits(__float_as_uint(q[k].w)), i + 3);
          uint64_t m01 = c0 > c1 ? c0 : c1, m23 = c2 > c3 ? c2 : c3;
          best = m01 > m23 ? m01 : m23;
        }
        for (int o = lpr / 2; o > 0; o >>= 1) {
          uint64_t w = __shfl_xor_sync(0xffffffffu, best, o, lpr);
          best = w > best ? w : best;
        }
        if (act[k] && lane_in_row == 0) out[oo[k]] = 0xffffffffu - (uint32_t)best;
      }
    }
    return;
  }
  for (uint64_t r0 = (uint64_t)blockIdx.x * rows_per_block; r0 < g.rows; r0 += row_stride) {
    const uint64_t r = r0 + threadIdx.x / lpr;
    const bool active = r < g.rows;
    uint64_t best = 0, xo = 0, oo = 0;
    if (active) {
      row_offsets(g, r, &xo, &oo);
      if (g.vec) {
        const float4* p = reinterpret_cast<const float4*>(x + xo);
        for (uint64_t v = lane_in_row; v < g.cols / 4; v += lpr) {
          float4 q = __ldcs(p + v);
          const uint64_t i = v * 4;
          uint64_t c0 = cand(key_of_bits(__float_as_uint(q.x)), i);
          uint64_t c1 = cand(key_of_bits(__float_as_uint(q.y)), i + 1);
          uint64_t c2 = cand(key_of_bits(__float_as_uint(q.z)), i + 2);
          uint64_t c3 = cand(key_of_bits(__float_as_uint(q.w)), i + 3);
          uint64_t m01 = c0 > c1 ? c0 : c1, m23 = c2 > c3 ? c2 : c3;
          uint64_t m = m01 > m23 ? m01 : m23;
          best = m > best ? m : best;
        }
      } else {
        for (uint64_t i = lane_in_row; i < g.cols; i += lpr) {
          uint64_t c = cand(key_of_bits(__float_as_uint(x[xo + i * g.col_stride])), i);
          best = c > best ? c : best;
        }
      }
    }
    // every lane of the warp reaches the shuffles (inactive rows carry the neutral 0)
    for (int o = lpr / 2; o > 0; o >>= 1) {
      uint64_t w = __shfl_xor_sync(0xffffffffu, best, o, lpr);
      best = w > best ? w : best;
    }
    (void)group_mask;
    if (active && lane_in_row == 0) out[oo] = 0xffffffffu - (uint32_t)best;
  }
}

// Rows of 16 to 512 floats (a power of two) in 16-byte aligned runs: L = cols / 16 lanes per
// row, each lane 4 float4s at columns 4 * (lane + L * j), two rows per thread in flight (8 loads).
// A lane scans its 16 values in increasing column order with a strict comparison, so it keeps the
// lowest index among equal keys and tracks the winner as a position 0..15 that becomes a column
// only once; NaN magnitudes clamp to 0x7f800001, above +inf and equal to one another, which
// orders exactly like kNanKey.  Only log2(L) shuffle levels remain per row.
template <int L>
__global__ void __launch_bounds__(kThreads) argmax_rows_vec_kernel(const float* __restrict__ x,
                                                                    uint32_t* __restrict__ out, RowGeom g) {
  constexpr int W = 4, R = 2;
  constexpr int kGroupRows = kThreads / L;  // rows per block per sub-pass
  const uint32_t lane = threadIdx.x % L;
  const uint64_t block_rows = (uint64_t)kGroupRows * R;
  for (uint64_t r0 = (uint64_t)blockIdx.x * block_rows; r0 < g.rows; r0 += (uint64_t)gridDim.x * block_rows) {
    float4 q[R][W];
    uint64_t oo[R];
    bool act[R];
#pragma unroll
    for (int k = 0; k < R; k++) {
      const uint64_t r = r0 + (uint64_t)k * kGroupRows + threadIdx.x / L;
      act[k] = r < g.rows;
      uint64_t xo = 0;
      oo[k] = 0;
      if (act[k]) row_offsets(g, r, &xo, &oo[k]);
      const float4* p = reinterpret_cast<const float4*>(x + xo) + lane;
#pragma unroll
      for (int j = 0; j < W; j++) q[k][j] = act[k] ? __ldcs(p + L * j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < R; k++) {
      uint32_t bk = 0, bp = 0;
#pragma unroll
      for (int j = 0; j < W; j++) {
        const float v[4] = {q[k][j].x, q[k][j].y, q[k][j].z, q[k][j].w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const uint32_t kk = min(__float_as_uint(v[e]) & 0x7fffffffu, 0x7f800001u);
          if (j == 0 && e == 0) {
            bk = kk;
          } else if (kk > bk) {
            bk = kk;
            bp = (uint32_t)(4 * j + e);
          }
        }
      }
      const uint32_t col = 4 * (lane + L * (bp >> 2)) + (bp & 3);
      uint64_t best = cand(bk, col);
#pragma unroll
      for (int o = L / 2; o > 0; o >>= 1) {
        const uint64_t w = __shfl_xor_sync(0xffffffffu, best, o, L);
        best = w > best ? w : best;
      }
      if (act[k] && lane == 0) out[oo[k]] = 0xffffffffu - (uint32_t)best;
    }
  }
}

lc_status check_out_one(const lc_view& out) {
  using namespace lc;
  if (out.dtype != LC_U32) return fail(LC_ERR_INVALID_ARGUMENT, "argmax output must be u32");
  if (out.rank > 1 || numel(out) != 1)
    return fail(LC_ERR_INVALID_ARGUMENT, "argmax output must hold one element");
  return LC_OK;
}

template <int KIND>
lc_status argmax_1d(lc_context* ctx, void* stream, const lc_view* xp, const lc_view* outp) {
  using namespace lc;
  if (ctx == nullptr || xp == nullptr || outp == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  const lc_view& x = *xp;
  const lc_view& out = *outp;
  // src/ops/argmax.rs:153-179 `encode` order
  if (x.rank != 1) return fail(LC_ERR_INVALID_ARGUMENT, "argmax input must be rank 1");
  const uint64_t n = x.shape[0];
  if (n == 0) return fail(LC_ERR_INVALID_ARGUMENT, "argmax input is empty");
  if (n > 0xffffffffull) return fail(LC_ERR_INVALID_ARGUMENT, "argmax input length exceeds u32::MAX");
  lc_status st = validate(x, "x");
  if (!st) st = validate(out, "out");
  if (st) return st;
  if ((KIND == 0 && x.dtype != LC_F32) || (KIND != 0 && x.dtype != LC_C32))
    return fail(LC_ERR_INVALID_ARGUMENT, KIND == 0 ? "argmax input must be f32" : "argmax_complex input must be complex f32");
  if ((st = check_out_one(out))) return st;
  if (may_overlap(x, out)) return fail(LC_ERR_OVERLAP, "argmax output overlaps its input");
  cudaStream_t s = stream_of(ctx, stream);
  const float* xb = static_cast<const float*>(x.data);
  uint32_t* ob = static_cast<uint32_t*>(out.data) + out.offset;
  if (n <= kSinglePassMax) {
    argmax_pass1<KIND><<<1, kThreads, 0, s>>>(xb, x.offset, x.strides[0], n, n, nullptr, ob);
    record_launch(ctx, "argmax_single");
  } else {
    const uint64_t groups =
        std::min<uint64_t>(kMaxGroups, std::max<uint64_t>(1, (n + kThreads * kItemsPerThread - 1) / (kThreads * kItemsPerThread)));
    const uint64_t chunk = (n + groups - 1) / groups;
    uint64_t* partials = nullptr;
    if ((st = scratch_alloc(ctx, s, sizeof(uint64_t) * groups, (void**)&partials))) return st;
    argmax_pass1<KIND><<<(unsigned)groups, kThreads, 0, s>>>(xb, x.offset, x.strides[0], n, chunk, partials, nullptr);
    record_launch(ctx, "argmax_partial");
    argmax_final<<<1, kThreads, 0, s>>>(partials, (int)groups, ob);
    record_launch(ctx, "argmax_final");
    scratch_free(partials, s);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
  return LC_OK;
}

}  // namespace

using namespace lc;

extern "C" {

lc_status lc_encode_argmax(lc_context* ctx, void* stream, const lc_view* x, const lc_view* out) {
  return argmax_1d<0>(ctx, stream, x, out);
}

lc_status lc_argmax(lc_context* ctx, const lc_view* x, const lc_view* out) {
  lc_status st = lc_encode_argmax(ctx, nullptr, x, out);
  return st ? st : lc_sync(ctx, nullptr);
}

lc_status lc_encode_argmax_complex(lc_context* ctx, void* stream, const lc_view* x, int32_t magnitude,
                                   const lc_view* out) {
  if (magnitude == 0) return argmax_1d<1>(ctx, stream, x, out);
  if (magnitude == 1) return argmax_1d<2>(ctx, stream, x, out);
  return fail(LC_ERR_INVALID_ARGUMENT, "magnitude is 0 (L1) or 1 (Hypot)");
}

lc_status lc_encode_argmax_rows(lc_context* ctx, void* stream, const lc_view* xp, const lc_view* outp) {
  if (ctx == nullptr || xp == nullptr || outp == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  const lc_view& x = *xp;
  const lc_view& out = *outp;
  lc_status st = validate(x, "x");
  if (!st) st = validate(out, "out");
  if (st) return st;
  if (x.dtype != LC_F32) return fail(LC_ERR_INVALID_ARGUMENT, "argmax input must be f32");
  if (out.dtype != LC_U32) return fail(LC_ERR_INVALID_ARGUMENT, "argmax output must be u32");
  if (x.rank < 1) return fail(LC_ERR_INVALID_ARGUMENT, "argmax_rows needs rank >= 1");
  if (out.rank != x.rank - 1 || memcmp(out.shape, x.shape, sizeof(uint64_t) * out.rank) != 0)
    return fail(LC_ERR_INVALID_ARGUMENT, "argmax_rows output shape must be the input's leading shape");
  const uint64_t cols = x.shape[x.rank - 1];
  if (cols == 0) return fail(LC_ERR_INVALID_ARGUMENT, "argmax rows are empty");
  if (cols > 0xffffffffull) return fail(LC_ERR_INVALID_ARGUMENT, "argmax row length exceeds u32::MAX");
  if (may_overlap(x, out)) return fail(LC_ERR_OVERLAP, "argmax output overlaps its input");
  if (is_empty(out)) return LC_OK;
  if (!is_injective(out)) return fail(LC_ERR_INVALID_ARGUMENT, "argmax output is not injective");
  RowGeom g{};
  g.rank = out.rank;
  g.rows = numel(out);
  g.cols = cols;
  g.col_stride = x.strides[x.rank - 1];
  g.x_off = x.offset;
  g.o_off = out.offset;
  for (int d = 0; d < out.rank; d++) {
    g.shape[d] = out.shape[d];
    g.xs[d] = x.strides[d];
    g.os[d] = out.strides[d];
  }
  // leading axes that step uniformly in both x and out (row r at r * stride) collapse to one
  {
    bool uniform = out.rank >= 1;
    for (int d = 0; d + 1 < out.rank && uniform; d++)
      if (x.strides[d] != x.strides[d + 1] * out.shape[d + 1] || out.strides[d] != out.strides[d + 1] * out.shape[d + 1])
        uniform = false;
    if (uniform && out.rank > 1) {
      g.rank = 1;
      g.shape[0] = g.rows;
      g.xs[0] = x.strides[out.rank - 1];
      g.os[0] = out.strides[out.rank - 1];
    }
  }
  bool vec = g.col_stride == 1 && cols % 4 == 0 && (reinterpret_cast<uintptr_t>(x.data) + x.offset * 4) % 16 == 0;
  for (int d = 0; d < out.rank && vec; d++)
    if (out.shape[d] > 1 && (x.strides[d] * 4) % 16 != 0) vec = false;
  g.vec = vec ? 1 : 0;
  cudaStream_t s = stream_of(ctx, stream);
  if (vec && cols >= 16 && cols <= 512 && (cols & (cols - 1)) == 0) {
    const int L = (int)(cols / 16);
    const uint64_t rows_per_pass = (uint64_t)(kThreads / L) * 2;
    const float* xp = static_cast<const float*>(x.data);
    uint32_t* op = static_cast<uint32_t*>(out.data);
    // one wave of resident blocks, each looping over its share of the rows
    auto launch = [&](auto lanes) {
      constexpr int kL = decltype(lanes)::value;
      static const int resident = [] {
        int b = 0;
        return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, argmax_rows_vec_kernel<kL>, kThreads, 0) == cudaSuccess && b > 0
                   ? b : 1;
      }();
      const uint64_t blocks = std::min<uint64_t>((g.rows + rows_per_pass - 1) / rows_per_pass,
                                                 (uint64_t)ctx->sm_count * resident);
      argmax_rows_vec_kernel<kL><<<(unsigned)std::max<uint64_t>(blocks, 1), kThreads, 0, s>>>(xp, op, g);
    };
    switch (L) {
      case 1: launch(std::integral_constant<int, 1>{}); break;
      case 2: launch(std::integral_constant<int, 2>{}); break;
      case 4: launch(std::integral_constant<int, 4>{}); break;
      case 8: launch(std::integral_constant<int, 8>{}); break;
      case 16: launch(std::integral_constant<int, 16>{}); break;
      default: launch(std::integral_constant<int, 32>{}); break;
    }
    record_launch(ctx, "argmax_rows");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "argmax_rows launch");
    return LC_OK;
  }
  int lpr = 1;
  const uint64_t per_lane_items = vec ? cols / 4 : cols;
  while (lpr < 32 && (uint64_t)lpr * 2 <= per_lane_items) lpr *= 2;
  const uint64_t rows_per_block = kThreads / lpr;
  const uint64_t blocks = std::min<uint64_t>((g.rows + rows_per_block - 1) / rows_per_block, (uint64_t)ctx->sm_count * 16);
  argmax_rows_kernel<<<(unsigned)std::max<uint64_t>(blocks, 1), kThreads, 0, s>>>(
      static_cast<const float*>(x.data), static_cast<uint32_t*>(out.data), g, lpr);
  record_launch(ctx, "argmax_rows");
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "argmax_rows launch");
  return LC_OK;
}

}  // extern "C"
