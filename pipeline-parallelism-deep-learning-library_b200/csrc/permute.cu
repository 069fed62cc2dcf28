// permute.cu -- strided copies: materialize / conjugate / adjoint (src/ops/permutation.rs) and
// pack / concat (src/ops/slicing.rs).
//
// One engine serves every op: the two views are merged jointly (axes contiguous in both fold
// together), then the cheapest kernel that fits runs:
//   rows      both views unit-stride on the same axis: each row moves as 16/8/4/2-byte words,
//             the widest that every row start and length allow; a warp covers whole rows, so
//             every load and store instruction is fully coalesced;
//   transpose the source is unit-stride on axis a and the destination on axis b != a: 64x64
//             4-byte (or 32x32 8-byte) tiles staged through padded shared memory, 16-byte
//             vectors on both global sides when the tile is interior and aligned;
//   scalar    anything else: one element per thread, mixed-radix decode.
// Index decode uses precomputed 32-bit magic divisors when every index fits in 32 bits.
// Bits move untouched (NaN payloads and -0 survive); `conj` flips the sign bit of the
// imaginary word of 8-byte complex elements.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "internal.h"

namespace {

// Unsigned 32-bit division by an invariant divisor (Granlund & Montgomery 1994, fig. 4.1).
struct FastDiv {
  uint32_t d, m, s1, s2;
};

FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{};
  f.d = d;
  uint32_t l = 0;
  while ((1ull << l) < d) l++;
  f.m = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
  f.s1 = l > 0 ? 1 : 0;
  f.s2 = l > 0 ? l - 1 : 0;
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  uint32_t t = __umulhi(f.m, n);
  return (t + ((n - t) >> f.s1)) >> f.s2;
}

constexpr int R = LC_MAX_RANK;

struct Geom {
  int rank;  // axes decoded per work item
  uint64_t shape[R];
  uint64_t ss[R];  // source strides (elements)
  uint64_t ds[R];  // destination strides (elements)
  FastDiv div[R];
  uint64_t src_off, dst_off;
  uint64_t count;  // work items
  // rows kernel
  uint64_t row_words;   // words per row
  uint32_t words_shift;  // log2(words per row) when a power of two, else 0xffffffff
  FastDiv row_div;
  // transpose kernel
  uint64_t ext_a, ext_b, src_stride_b, dst_stride_a;
  uint32_t tiles_a, tiles_b;
  int conj;
  int small;  // every index fits in 32 bits
};

template <bool SMALL>
__device__ __forceinline__ void decode(const Geom& g, uint64_t i, uint64_t* so, uint64_t* dof) {
  uint64_t s = 0, d = 0;
  if (SMALL) {
    uint32_t r = (uint32_t)i;
    for (int a = g.rank - 1; a >= 0; a--) {
      uint32_t q = fdiv(r, g.div[a]);
      uint32_t c = r - q * g.div[a].d;
      r = q;
      s += (uint64_t)c * g.ss[a];
      d += (uint64_t)c * g.ds[a];
    }
  } else {
    for (int a = g.rank - 1; a >= 0; a--) {
      uint64_t n = g.shape[a];
      uint64_t c = i % n;
      i /= n;
      s += c * g.ss[a];
      d += c * g.ds[a];
    }
  }
  *so = s;
  *dof = d;
}

template <typename W>
__device__ __forceinline__ W conj_word(W v, int conj) {
  if constexpr (sizeof(W) == 8) {
    if (conj) {
      uint2 u = *reinterpret_cast<uint2*>(&v);
      u.y ^= 0x80000000u;
      return *reinterpret_cast<W*>(&u);
    }
  }
  return v;
}

// ---- scalar gather ----------------------------------------------------------------------------
template <typename E, bool SMALL>
__global__ void __launch_bounds__(256) copy_scalar_kernel(const E* __restrict__ src, E* __restrict__ dst, Geom g) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < g.count; i += stride) {
    uint64_t so, dof;
    decode<SMALL>(g, i, &so, &dof);
    dst[g.dst_off + dof] = conj_word(src[g.src_off + so], g.conj);
  }
}

// ---- rows ---------------------------------------------------------------------------------------
// Work item = one word of one row.  Row r's outer offsets come from decoding r over the outer axes
// (g.rank of them); the words of a row are contiguous on both sides.  src/dst are word pointers
// already advanced by the byte offsets.  Each thread moves kRowUnroll words per pass, all loads
// before any store, so that several loads per thread are in flight (one at a time left the copy
// latency-bound).
constexpr int kRowUnroll = 4;

// Streaming row load.  16-byte words carry an L2 fetch-size hint of 64 bytes: a sliced row that
// covers half of each of two 128-byte lines (32 floats from byte 64 of a 256-byte row) otherwise
// pulls both whole lines from DRAM, twice the bytes the copy uses.
template <typename Wd>
__device__ __forceinline__ Wd ld_row_word(const Wd* p) {
  if constexpr (sizeof(Wd) == 16) {
    uint4 v;
    asm volatile("ld.global.cs.L2::64B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return *reinterpret_cast<Wd*>(&v);
  } else {
    return __ldcs(p);
  }
}

template <typename Wd, bool SMALL>
__global__ void __launch_bounds__(256) copy_rows_kernel(const Wd* __restrict__ src, Wd* __restrict__ dst, Geom g) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i0 = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i0 < g.count; i0 += stride * kRowUnroll) {
    Wd v[kRowUnroll];
    uint64_t at[kRowUnroll];
#pragma unroll
    for (int u = 0; u < kRowUnroll; u++) {
      const uint64_t i = i0 + u * stride;
      if (i >= g.count) continue;
      uint64_t row, col;
      if (g.words_shift != 0xffffffffu) {
        row = i >> g.words_shift;
        col = i & (g.row_words - 1);
      } else if (SMALL) {
        uint32_t q = fdiv((uint32_t)i, g.row_div);
        row = q;
        col = (uint32_t)i - q * g.row_div.d;
      } else {
        row = i / g.row_words;
        col = i - row * g.row_words;
      }
      uint64_t so, dof;
      decode<SMALL>(g, row, &so, &dof);
      v[u] = ld_row_word(src + so + col);
      at[u] = dof + col;
    }
#pragma unroll
    for (int u = 0; u < kRowUnroll; u++)
      if (i0 + u * stride < g.count) dst[at[u]] = conj_word(v[u], g.conj);
  }
}

// ---- tiled transpose ------------------------------------------------------------------------------
// Source unit-stride along a, destination unit-stride along b.  Tile = T x T elements with
// T * sizeof(E) = 256 bytes.  Block (x: b tile, y: a tile, z: outer) of 256 threads.
template <typename E, bool SMALL>
__global__ void __launch_bounds__(256) transpose_kernel(const E* __restrict__ src, E* __restrict__ dst, Geom g) {
  constexpr int T = 256 / sizeof(E);   // 64 (4-byte) or 32 (8-byte) or 128 (2-byte)
  constexpr int V = 16 / sizeof(E);    // elements per 16-byte vector
  constexpr int VPR = T / V;           // vectors per tile row (16)
  constexpr int RPP = 256 / VPR;       // tile rows per pass (16)
  __shared__ E tile[T][T + (sizeof(E) == 8 ? 1 : (sizeof(E) == 4 ? 1 : 2))];
  const uint64_t a0 = (uint64_t)blockIdx.y * T;
  const uint64_t b0 = (uint64_t)blockIdx.x * T;
  for (uint64_t o = blockIdx.z; o < g.count; o += gridDim.z) {
    uint64_t so, dof;
    decode<SMALL>(g, o, &so, &dof);
    const E* s = src + g.src_off + so;
    E* d = dst + g.dst_off + dof;
    const bool full_a = a0 + T <= g.ext_a, full_b = b0 + T <= g.ext_b;
    const int tx = threadIdx.x % VPR, ty = threadIdx.x / VPR;
    // load: tile[bb][aa] = src[(a0+aa) + (b0+bb)*stride_b].  A whole, 16-byte aligned tile
    // issues all of a thread's T / RPP vector loads before its first shared-memory store.
    const bool whole = full_a && b0 + T <= g.ext_b &&
                       reinterpret_cast<uintptr_t>(s + b0 * g.src_stride_b + a0) % 16 == 0 &&
                       (g.src_stride_b * sizeof(E)) % 16 == 0;
    if (whole) {
      uint4 v[T / RPP];
#pragma unroll
      for (int k = 0; k < T / RPP; k++)
        v[k] = __ldcs(reinterpret_cast<const uint4*>(s + (b0 + ty + k * RPP) * g.src_stride_b + a0) + tx);
#pragma unroll
      for (int k = 0; k < T / RPP; k++) {
        const E* e = reinterpret_cast<const E*>(&v[k]);
#pragma unroll
        for (int u = 0; u < V; u++) tile[ty + k * RPP][tx * V + u] = e[u];
      }
    }
    for (int bb = ty; bb < T && !whole; bb += RPP) {
      const uint64_t b = b0 + bb;
      const E* row = s + b * g.src_stride_b + a0;
      if (full_a && b < g.ext_b && (reinterpret_cast<uintptr_t>(row) % 16 == 0)) {
        uint4 v = __ldcs(reinterpret_cast<const uint4*>(row) + tx);
        const E* e = reinterpret_cast<const E*>(&v);
#pragma unroll
        for (int u = 0; u < V; u++) tile[bb][tx * V + u] = e[u];
      } else {
#pragma unroll
        for (int u = 0; u < V; u++) {
          const uint64_t aa = (uint64_t)tx * V + u;
          if (b < g.ext_b && a0 + aa < g.ext_a) tile[bb][aa] = row[aa];
        }
      }
    }
    __syncthreads();
    // store: dst[(a0+aa)*stride_a + b0 + bb] = tile[bb][aa]
    for (int aa = ty; aa < T; aa += RPP) {
      const uint64_t a = a0 + aa;
      E* row = d + a * g.dst_stride_a + b0;
      if (full_b && a < g.ext_a && (reinterpret_cast<uintptr_t>(row) % 16 == 0)) {
        uint4 v;
        E* e = reinterpret_cast<E*>(&v);
#pragma unroll
        for (int u = 0; u < V; u++) e[u] = conj_word(tile[tx * V + u][aa], g.conj);
        __stcs(reinterpret_cast<uint4*>(row) + tx, v);
      } else {
#pragma unroll
        for (int u = 0; u < V; u++) {
          const uint64_t bb = (uint64_t)tx * V + u;
          if (a < g.ext_a && b0 + bb < g.ext_b) row[bb] = conj_word(tile[bb][aa], g.conj);
        }
      }
    }
    __syncthreads();
  }
}

template <int EB>
struct Elem;
template <>
struct Elem<1> { using T = uint8_t; };
template <>
struct Elem<2> { using T = uint16_t; };
template <>
struct Elem<4> { using T = uint32_t; };
template <>
struct Elem<8> { using T = uint2; };
template <>
struct Elem<16> { using T = uint4; };

unsigned grid_cap(lc_context* ctx, uint64_t items, unsigned block, unsigned per_sm = 16) {
  uint64_t want = (items + block - 1) / block;
  uint64_t cap = (uint64_t)ctx->sm_count * per_sm;
  return (unsigned)std::max<uint64_t>(1, std::min(want, cap));
}

void set_divs(Geom& g) {
  for (int a = 0; a < g.rank; a++) g.div[a] = make_fastdiv((uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(g.shape[a], 0xffffffffu)));
}

template <int EB>
lc_status launch_scalar(lc_context* ctx, cudaStream_t s, const void* src, void* dst, Geom& g) {
  using E = typename Elem<EB>::T;
  set_divs(g);
  unsigned grid = grid_cap(ctx, g.count, 256);
  if (g.small)
    copy_scalar_kernel<E, true><<<grid, 256, 0, s>>>((const E*)src, (E*)dst, g);
  else
    copy_scalar_kernel<E, false><<<grid, 256, 0, s>>>((const E*)src, (E*)dst, g);
  lc::record_launch(ctx, "strided_copy_scalar");
  return LC_OK;
}

template <typename Wd>
lc_status launch_rows(lc_context* ctx, cudaStream_t s, const uint8_t* src, uint8_t* dst, Geom& g) {
  set_divs(g);
  unsigned grid = grid_cap(ctx, g.count, 256);
  if (g.small)
    copy_rows_kernel<Wd, true><<<grid, 256, 0, s>>>((const Wd*)src, (Wd*)dst, g);
  else
    copy_rows_kernel<Wd, false><<<grid, 256, 0, s>>>((const Wd*)src, (Wd*)dst, g);
  lc::record_launch(ctx, sizeof(Wd) == 16 ? "strided_copy_rows16" : sizeof(Wd) == 8 ? "strided_copy_rows8"
                                                                     : sizeof(Wd) == 4 ? "strided_copy_rows4"
                                                                                        : "strided_copy_rows2");
  return LC_OK;
}

template <int EB>
lc_status launch_transpose(lc_context* ctx, cudaStream_t s, const void* src, void* dst, Geom& g) {
  using E = typename Elem<EB>::T;
  constexpr int T = 256 / EB;
  set_divs(g);
  uint64_t ta = (g.ext_a + T - 1) / T, tb = (g.ext_b + T - 1) / T;
  if (ta > 65535 || tb > 0x7fffffffull) return lc::fail(LC_ERR_INVALID_ARGUMENT, "transpose extent too large");
  dim3 grid((unsigned)tb, (unsigned)ta, (unsigned)std::min<uint64_t>(std::max<uint64_t>(g.count, 1), 65535));
  if (g.small)
    transpose_kernel<E, true><<<grid, 256, 0, s>>>((const E*)src, (E*)dst, g);
  else
    transpose_kernel<E, false><<<grid, 256, 0, s>>>((const E*)src, (E*)dst, g);
  lc::record_launch(ctx, "strided_copy_transpose");
  return LC_OK;
}

}  // namespace

namespace lc {

lc_status launch_strided_copy(lc_context* ctx, cudaStream_t s, const void* src, uint64_t src_off, void* dst,
                              uint64_t dst_off, int rank, const uint64_t* shape, const uint64_t* src_strides,
                              const uint64_t* dst_strides, size_t eb, bool conj) {
  // Joint merge: drop unit axes, fold an axis into its outer neighbour when both views are
  // contiguous across them.
  std::vector<uint64_t> sh, ss, ds;
  uint64_t count = 1;
  for (int d = 0; d < rank; d++) {
    count *= shape[d];
    if (shape[d] == 1) continue;
    if (!sh.empty() && ss.back() == src_strides[d] * shape[d] && ds.back() == dst_strides[d] * shape[d]) {
      sh.back() *= shape[d];
      ss.back() = src_strides[d];
      ds.back() = dst_strides[d];
      continue;
    }
    sh.push_back(shape[d]);
    ss.push_back(src_strides[d]);
    ds.push_back(dst_strides[d]);
  }
  if (count == 0) return LC_OK;
  if (sh.empty()) {
    sh.push_back(1);
    ss.push_back(1);
    ds.push_back(1);
  }
  const int r = (int)sh.size();
  Geom g{};
  g.conj = conj ? 1 : 0;
  g.src_off = src_off;
  g.dst_off = dst_off;
  uint64_t smax = src_off, dmax = dst_off;
  for (int d = 0; d < r; d++) {
    smax += (sh[d] - 1) * ss[d];
    dmax += (sh[d] - 1) * ds[d];
  }
  g.small = (count < (1ull << 32) && smax < (1ull << 32) && dmax < (1ull << 32)) ? 1 : 0;

  // rows: both unit-stride on the last merged axis.
  if (ss[r - 1] == 1 && ds[r - 1] == 1 && eb >= 2) {
    const uint64_t inner = sh[r - 1];
    const uint8_t* sb = static_cast<const uint8_t*>(src) + src_off * eb;
    uint8_t* db = static_cast<uint8_t*>(dst) + dst_off * eb;
    // The widest word (16, 8, 4 or 2 bytes) that every row start and the row length allow.
    auto ok = [&](size_t width) {
      if ((reinterpret_cast<uintptr_t>(sb) % width) || (reinterpret_cast<uintptr_t>(db) % width)) return false;
      if ((inner * eb) % width) return false;
      for (int d = 0; d < r - 1; d++)
        if ((ss[d] * eb) % width || (ds[d] * eb) % width) return false;
      return true;
    };
    size_t w = 16;
    while (w > 2 && !ok(w)) w /= 2;
    if (conj) w = 8;  // conjugation flips the imaginary word of whole 8-byte complex elements
    if (ok(w)) {
      g.rank = r - 1;
      for (int d = 0; d < r - 1; d++) {
        g.shape[d] = sh[d];
        g.ss[d] = ss[d] * eb / w;
        g.ds[d] = ds[d] * eb / w;
      }
      g.row_words = inner * eb / w;
      g.count = count / inner * g.row_words;
      g.words_shift = 0xffffffffu;
      if ((g.row_words & (g.row_words - 1)) == 0) {
        uint32_t sh2 = 0;
        while ((1ull << sh2) < g.row_words) sh2++;
        g.words_shift = sh2;
      }
      g.row_div = make_fastdiv((uint32_t)std::min<uint64_t>(g.row_words, 0xffffffffu));
      if (g.count >= (1ull << 32)) g.small = 0;
      g.src_off = g.dst_off = 0;
      switch (w) {
        case 16: return launch_rows<uint4>(ctx, s, sb, db, g);
        case 8: return launch_rows<uint2>(ctx, s, sb, db, g);
        case 4: return launch_rows<uint32_t>(ctx, s, sb, db, g);
        default: return launch_rows<uint16_t>(ctx, s, sb, db, g);
      }
    }
  }

  // transpose: source unit-stride on axis a, destination unit-stride on axis b != a.
  int a = -1, b = -1;
  for (int d = 0; d < r; d++) {
    if (ss[d] == 1 && a < 0) a = d;
    if (ds[d] == 1 && b < 0) b = d;
  }
  if (a >= 0 && b >= 0 && a != b && (eb == 4 || eb == 8 || eb == 2) && sh[a] > 1 && sh[b] > 1) {
    g.rank = 0;
    g.count = 1;
    for (int d = 0; d < r; d++) {
      if (d == a || d == b) continue;
      g.shape[g.rank] = sh[d];
      g.ss[g.rank] = ss[d];
      g.ds[g.rank] = ds[d];
      g.rank++;
      g.count *= sh[d];
    }
    g.ext_a = sh[a];
    g.ext_b = sh[b];
    g.src_stride_b = ss[b];
    g.dst_stride_a = ds[a];
    switch (eb) {
      case 2: return launch_transpose<2>(ctx, s, src, dst, g);
      case 4: return launch_transpose<4>(ctx, s, src, dst, g);
      default: return launch_transpose<8>(ctx, s, src, dst, g);
    }
  }

  g.rank = r;
  for (int d = 0; d < r; d++) {
    g.shape[d] = sh[d];
    g.ss[d] = ss[d];
    g.ds[d] = ds[d];
  }
  g.count = count;
  switch (eb) {
    case 1: return launch_scalar<1>(ctx, s, src, dst, g);
    case 2: return launch_scalar<2>(ctx, s, src, dst, g);
    case 4: return launch_scalar<4>(ctx, s, src, dst, g);
    case 8: return launch_scalar<8>(ctx, s, src, dst, g);
    case 16: return launch_scalar<16>(ctx, s, src, dst, g);
    default: return fail(LC_ERR_INVALID_ARGUMENT, "element size must be 1, 2, 4, 8 or 16 bytes");
  }
}

}  // namespace lc

using namespace lc;

namespace {

lc_status finish_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return LC_OK;
}

// src/ops/permutation.rs:163-270 `encode_gather` checks, then the copy engine.
lc_status gather(lc_context* ctx, void* stream, const lc_view* srcp, const lc_view* dstp, bool conj) {
  if (ctx == nullptr || srcp == nullptr || dstp == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  const lc_view& src = *srcp;
  const lc_view& dst = *dstp;
  lc_status st = validate(src, "source");
  if (st) return st;
  if ((st = validate(dst, "destination"))) return st;
  size_t eb = dtype_size(src.dtype);
  if (src.dtype != dst.dtype) return fail(LC_ERR_INVALID_ARGUMENT, "source and destination element types differ");
  if (!(src.dtype == LC_F32 || src.dtype == LC_U32 || src.dtype == LC_I32 || src.dtype == LC_C32))
    return fail(LC_ERR_INVALID_ARGUMENT, "permutation elements are f32, u32, i32 or complex f32");
  if (src.rank != dst.rank || memcmp(src.shape, dst.shape, sizeof(uint64_t) * src.rank) != 0)
    return fail(LC_ERR_INVALID_ARGUMENT, "destination shape does not match source shape");
  uint64_t dense[R];
  row_major_strides(dst.shape, dst.rank, dense);
  for (int d = 0; d < dst.rank; d++)
    if (dst.shape[d] != 1 && dst.strides[d] != dense[d])
      return fail(LC_ERR_INVALID_ARGUMENT, "destination must be contiguous row-major");
  if (may_overlap(src, dst)) return fail(LC_ERR_OVERLAP, "destination overlaps the source");
  if (is_empty(src)) return LC_OK;
  cudaStream_t s = stream_of(ctx, stream);
  st = launch_strided_copy(ctx, s, src.data, src.offset, dst.data, dst.offset, src.rank, src.shape, src.strides,
                           dst.strides, eb, conj && src.dtype == LC_C32);
  if (st) return st;
  return finish_launch("materialize");
}

}  // namespace

extern "C" {

lc_status lc_encode_materialize(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst) {
  return gather(ctx, stream, src, dst, false);
}

lc_status lc_materialize(lc_context* ctx, const lc_view* src, const lc_view* dst) {
  lc_status st = lc_encode_materialize(ctx, nullptr, src, dst);
  return st ? st : lc_sync(ctx, nullptr);
}

lc_status lc_encode_conjugate(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst) {
  return gather(ctx, stream, src, dst, true);
}

lc_status lc_encode_adjoint(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst) {
  if (src == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (src->rank < 2)
    return fail(LC_ERR_INVALID_ARGUMENT, "adjoint needs at least 2 axes, got " + std::to_string(src->rank));
  int32_t perm[R];
  for (int i = 0; i < src->rank; i++) perm[i] = i;
  std::swap(perm[src->rank - 2], perm[src->rank - 1]);
  lc_view t;
  lc_status st = lc_permute_view(src, perm, src->rank, &t);
  if (st) return st;
  return gather(ctx, stream, &t, dst, true);
}

// src/ops/slicing.rs:523-584 `encode_pack`.
lc_status lc_encode_pack(lc_context* ctx, void* stream, const lc_view* srcp, const lc_view* dstp) {
  if (ctx == nullptr || srcp == nullptr || dstp == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  const lc_view& src = *srcp;
  const lc_view& dst = *dstp;
  lc_status st = validate(src, "source");
  if (st) return st;
  if ((st = validate(dst, "destination"))) return st;
  size_t eb = dtype_size(src.dtype);
  if (dtype_size(dst.dtype) != eb) return fail(LC_ERR_INVALID_ARGUMENT, "element sizes differ");
  if (!(eb == 2 || eb == 4 || eb == 8 || eb == 16))
    return fail(LC_ERR_INVALID_ARGUMENT, "element size " + std::to_string(eb) + " is not 2, 4, 8, or 16 bytes");
  if (src.rank != dst.rank || memcmp(src.shape, dst.shape, sizeof(uint64_t) * src.rank) != 0)
    return fail(LC_ERR_INVALID_ARGUMENT, "destination shape does not match source shape");
  if (may_overlap(src, dst)) return fail(LC_ERR_OVERLAP, "destination overlaps the source");
  if (is_empty(src)) return LC_OK;
  if (!is_injective(dst))
    return fail(LC_ERR_INVALID_ARGUMENT, "destination layout aliases an element, so a parallel store would race");
  cudaStream_t s = stream_of(ctx, stream);
  st = launch_strided_copy(ctx, s, src.data, src.offset, dst.data, dst.offset, src.rank, src.shape, src.strides,
                           dst.strides, eb, false);
  if (st) return st;
  return finish_launch("pack");
}

lc_status lc_pack(lc_context* ctx, const lc_view* src, const lc_view* dst) {
  lc_status st = lc_encode_pack(ctx, nullptr, src, dst);
  return st ? st : lc_sync(ctx, nullptr);
}

// src/ops/slicing.rs:598-753 `encode_concat`: parts laid out in order along `axis`.
lc_status lc_encode_concat(lc_context* ctx, void* stream, const lc_view* parts, int32_t n_parts, int32_t axis,
                           const lc_view* dstp) {
  if (ctx == nullptr || dstp == nullptr || (parts == nullptr && n_parts > 0))
    return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (n_parts <= 0) return fail(LC_ERR_INVALID_ARGUMENT, "concat needs at least one part");
  if (n_parts > LC_MAX_CONCAT_PARTS)
    return fail(LC_ERR_INVALID_ARGUMENT, std::to_string(n_parts) + " parts exceeds the limit of 16");
  const lc_view& dst = *dstp;
  lc_status st = validate(dst, "destination");
  if (st) return st;
  size_t eb = dtype_size(dst.dtype);
  if (!(eb == 2 || eb == 4 || eb == 8 || eb == 16))
    return fail(LC_ERR_INVALID_ARGUMENT, "element size is not 2, 4, 8, or 16 bytes");
  if (dst.rank == 0 || axis < 0 || axis >= dst.rank)
    return fail(LC_ERR_INVALID_ARGUMENT, "axis " + std::to_string(axis) + " is out of range");
  uint64_t sum = 0;
  for (int i = 0; i < n_parts; i++) {
    const lc_view& p = parts[i];
    if ((st = validate(p, "part"))) return st;
    if (dtype_size(p.dtype) != eb) return fail(LC_ERR_INVALID_ARGUMENT, "part element size differs");
    if (p.rank != dst.rank) return fail(LC_ERR_INVALID_ARGUMENT, "part " + std::to_string(i) + " rank differs");
    for (int d = 0; d < dst.rank; d++)
      if (d != axis && p.shape[d] != dst.shape[d])
        return fail(LC_ERR_INVALID_ARGUMENT, "part " + std::to_string(i) + " extent differs on axis " + std::to_string(d));
    if (may_overlap(p, dst)) return fail(LC_ERR_OVERLAP, "destination overlaps part " + std::to_string(i));
    sum += p.shape[axis];
  }
  if (sum != dst.shape[axis]) return fail(LC_ERR_INVALID_ARGUMENT, "parts do not cover the destination extent");
  if (is_empty(dst)) return LC_OK;
  if (!is_injective(dst))
    return fail(LC_ERR_INVALID_ARGUMENT, "destination layout aliases an element, so a parallel store would race");
  cudaStream_t s = stream_of(ctx, stream);
  uint64_t prefix = 0;
  for (int i = 0; i < n_parts; i++) {
    const lc_view& p = parts[i];
    if (!is_empty(p)) {
      st = launch_strided_copy(ctx, s, p.data, p.offset, dst.data, dst.offset + prefix * dst.strides[axis], p.rank,
                               p.shape, p.strides, dst.strides, eb, false);
      if (st) return st;
    }
    prefix += p.shape[axis];
  }
  return finish_launch("concat");
}

}  // extern "C"
