// gemm_tc.cu -- the contraction's GEMM on sm_100a tensor cores.
//
// C[b] = alpha * A[b] @ B[b] + beta * C[b] for a batch of M x N x K products, every operand
// single-stride per group (the planner stages anything else first).
//
// Kernel (one persistent CTA per SM, warp-specialised):
//   warp 0      TMA producer: 128-byte-swizzled tiles of A (128 x BK) and B (BN x BK) into a
//               STAGES-deep shared-memory ring, completion on an mbarrier per stage;
//   warp 1      allocates TMEM (2 accumulators x BN f32 columns) and issues tcgen05.mma
//               (M=128, N=BN) from one thread; tcgen05.commit frees each stage and, after a
//               tile's last k block, hands the accumulator to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, alpha/beta (or a raw f32 split-K
//               partial), optional ReLU, store with C's strides; double-buffered accumulators
//               let tile i's epilogue overlap tile i+1's main loop;
//   warps 6-9   (3xTF32 only) split each staged f32 tile into tf32 hi (low 13 mantissa bits
//               cleared) and lo = x - hi, in place / into a second buffer; the MMA warp then
//               issues lo*hi + hi*lo + hi*hi.
// Operands may be K-major (K contiguous) or MN-major (M or N contiguous); both feed the
// tensor cores directly through the descriptors' major bits.  No TMA multicast anywhere: the
// same binary runs on 1 and on 8 GPUs.
// Every mbarrier wait is bounded (ptx.cuh); a timeout sets the context's device error word.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>

#include "activation.cuh"
#include "gemm.h"
#include "internal.h"
#include "ptx.cuh"

namespace {

constexpr int kBM = 128;
constexpr int kRowBytes = 128;  // one swizzle-128B row: 64 bf16/f16 or 32 f32 along the packed axis

struct KParams {
  int32_t M, N;
  int32_t k_tiles, kt_per_split, splits, batch;
  int32_t tiles_m, tiles_n;
  int32_t units;
  uint32_t a_mn, b_mn;
  uint32_t idesc;
  // epilogue
  int32_t c_dtype;  // LC_F32 / LC_BF16 / LC_F16
  int32_t relu;
  void* c;
  int64_t c_off, c_bs, c_ms, c_ns;
  float alpha, beta;
  float* partial;   // split-K: [splits][batch][M][N] raw partial sums
  int* counters;    // split-K fixup: one arrival counter per (batch, tile, epilogue warp), zero at launch
  int32_t fixup;    // 1: the last-arriving warp reduces in the kernel; 0: a separate reduce kernel does
  int32_t split_minor;  // unit u = tile * splits + split (CTA pairs); else u = split * tiles + tile
  int32_t a_once, b_once;  // the operand is read by exactly one CTA (one tile column / row): evict first
  int32_t prefetch;  // k-tiles of the once-read A operand requested into L2 ahead of the ring (0: none)
  int32_t vec;      // C's columns contiguous and every row start 16-byte aligned (C, aux and aux2)
  int32_t tvec;     // C's rows contiguous instead (swapped products), runs of 8 rows 16-byte aligned
  int* err;
  const void* aux;
  void* aux2;
  float lr;
  // 3xTF32: a unit whose operand tiles hold an infinity or NaN is recomputed exactly on the CUDA
  // cores from the operands as plain f32 arrays (element offsets applied): A (rows M) element
  // [b * fa_bs + m * fa_ms + k * fa_ks], B (rows N) element [b * fb_bs + n * fb_ns + k * fb_ks]
  const float* fa;
  const float* fb;
  int64_t fa_ms, fa_ks, fa_bs, fb_ns, fb_ks, fb_bs;
  int64_t K;
};

constexpr int kSmemMax = 232448;  // dynamic shared memory a CTA may opt in to on sm_100
constexpr int kPrefetchTiles = 0;  // default L2 prefetch distance of CTA-pair products, in k-tiles

template <int BN, bool TF32X3, bool PAIR = false, bool TWO_SM = false>
struct Cfg {
  static constexpr int EPR = TF32X3 ? 32 : 64;             // elements per 128-byte row
  static constexpr int BK = EPR;                           // K per stage
  static constexpr int UMMA_K = TF32X3 ? 8 : 16;           // K per instruction (32 bytes)
  static constexpr int KSTEPS = BK / UMMA_K;               // 4
  static constexpr int A_BYTES = kBM * kRowBytes;          // 16 KiB
  // TWO_SM: each CTA of the pair holds half of the tile's BN rows of B^T
  static constexpr int B_BYTES = (TWO_SM ? BN / 2 : BN) * kRowBytes;
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * (TF32X3 ? 2 : 1);
  // PAIR: the peer's raw partial of this CTA's column half lands here (f32, 128 x RECV_COLS), in
  // EXCH_ROUNDS rounds of RECV_COLS columns (two rounds for BN = 256, so that the ring keeps 4
  // stages of 48 KiB beside the buffer)
  static constexpr int RECV_COLS = BN / 2 < 64 ? BN / 2 : 64;
  static constexpr int EXCH_ROUNDS = (BN / 2) / RECV_COLS;
  static constexpr int RECV_BYTES = PAIR ? kBM * RECV_COLS * 4 : 0;
  static constexpr int STAGES_FIT = (kSmemMax - 1024 - 512 - RECV_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = PAIR ? (STAGES_FIT < 8 ? STAGES_FIT : 8) : 196608 / STAGE_BYTES;
  // 2 accumulators (+ the 3xTF32 running sum), rounded up to the power of two tcgen05.alloc takes
  static constexpr int TMEM_NEED = (TF32X3 ? 3 : 2) * BN;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                   : TMEM_NEED <= 256 ? 256 : 512;
  static_assert(TMEM_NEED <= 512, "TMEM holds 512 columns");
  // 3xTF32: 8 converter warps (two per SM sub-partition) hide the shared-memory latency that
  // one warp per sub-partition left exposed
  static constexpr int CONV_THREADS = TF32X3 ? 256 : 0;
  static constexpr int THREADS = 192 + CONV_THREADS;
  // k-tiles per accumulator hand-off: one per unit for 16-bit inputs; 2 (64 K values, 24 MMAs)
  // for 3xTF32, which bounds the truncation bias of the tensor core's f32 accumulation to
  // about 24 ulp-halves per chunk while the chunks themselves are summed round-to-nearest.
  static constexpr int KC = TF32X3 ? 2 : (1 << 30);
  static constexpr int BAR_BYTES = 8 * (3 * STAGES + 7) + 16 + 32;  // + 8 non-finite unit stamps
  // non-pair kernels: one 32 x 36 f32 tile per epilogue warp for coalesced row stores
  static constexpr int EPI_STAGE_BYTES = PAIR ? 0 : 4 * 32 * 36 * 4;
  static constexpr int SMEM = STAGES * STAGE_BYTES + ((BAR_BYTES + 15) / 16) * 16 + RECV_BYTES + EPI_STAGE_BYTES + 1024;
  static_assert(STAGES >= 2, "at least two stages");
  static_assert(SMEM <= kSmemMax, "shared memory budget");
  static_assert(!PAIR || (!TF32X3 && BN <= 256), "CTA pairs: 16-bit inputs, BN <= 256");
  static_assert(!PAIR || STAGES >= 4, "CTA pairs keep at least 4 stages in flight");
  static_assert(!TWO_SM || (!TF32X3 && BN == 256), "2-SM products: 16-bit inputs, BN = 256");
};

__device__ __forceinline__ void unit_coords(const KParams& p, int32_t u, int32_t* b, int32_t* split, int32_t* tm,
                                            int32_t* tn) {
  const int32_t per = p.tiles_m * p.tiles_n;
  int32_t t;
  if (p.split_minor) {
    const int32_t tt = u / p.splits;
    *split = u - tt * p.splits;
    *b = tt / per;
    t = tt - *b * per;
  } else {
    const int32_t bs = u / per;
    t = u - bs * per;
    *b = bs / p.splits;
    *split = bs - *b * p.splits;
  }
  // grouped raster: 8 M tiles share each sweep over N so concurrent CTAs reuse A and B panels in L2
  constexpr int32_t G = 8;
  const int32_t in_group = G * p.tiles_n;
  const int32_t group = t / in_group;
  const int32_t first_m = group * G;
  const int32_t gsize = min(p.tiles_m - first_m, G);
  const int32_t r = t - group * in_group;
  *tm = first_m + r % gsize;
  *tn = r / gsize;
}

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float x) {
  uint32_t bits = __float_as_uint(x);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
  uint32_t lsb = (bits >> 16) & 1u;
  return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}

__device__ __forceinline__ float load_c(const KParams& p, int64_t idx) {
  if (p.c_dtype == LC_F32) return static_cast<const float*>(p.c)[idx];
  const uint16_t h = static_cast<const uint16_t*>(p.c)[idx];
  if (p.c_dtype == LC_BF16) return __uint_as_float(((uint32_t)h) << 16);
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t to_half_bits(const KParams& p, float v) {
  return p.c_dtype == LC_BF16 ? f32_to_bf16_rne(v) : __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ float from_half_bits(const KParams& p, uint16_t h) {
  return p.c_dtype == LC_BF16 ? __uint_as_float(((uint32_t)h) << 16) : __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ void store_c(const KParams& p, int64_t idx, float v) {
  if (p.c_dtype == LC_F32) static_cast<float*>(p.c)[idx] = v;
  else static_cast<uint16_t*>(p.c)[idx] = to_half_bits(p, v);
}

__device__ __forceinline__ float finish(const KParams& p, float acc, float cold) {
  float v = __fmul_rn(p.alpha, acc);
  if (p.beta != 0.0f) v = __fadd_rn(v, __fmul_rn(p.beta, cold));
  if (p.relu) v = v > 0.0f ? v : 0.0f;
  return v;
}

// ---- epilogue variants ---------------------------------------------------------------------------
// EPI is a template parameter so that each kernel instance carries only its own epilogue:
//   0  C = alpha * acc + beta * C, optional ReLU; C f32 / bf16 / f16 with any strides;
//   1  C = alpha * acc where aux > 0, else +0 (aux: bf16 laid out like C) -- the ReLU derivative
//      fused into the data-gradient product;
//   2  master = master - lr * (alpha * acc), aux2 = bf16(master) (aux: f32 master, aux2: bf16 copy,
//      both laid out like C; C itself is unused) -- the SGD step fused into the weight gradient;
//   3  pre = alpha * acc + beta * C, aux2 = pre (when set), C = gelu(pre) -- a GELU layer's forward
//      (f32: C and aux2 f32);
//   4  C = (alpha * acc) * gelu'(aux) (aux: f32 pre-activation laid out like C) -- the data
//      gradient through a GELU layer's derivative (f32).
// `old` is what the variant reads before it writes: C (EPI 0 and 3, beta != 0), the mask (1),
// master (2), the pre-activation (4).

template <int EPI>
__device__ __forceinline__ float read_old(const KParams& p, int64_t idx) {
  if constexpr (EPI == 0 || EPI == 3) return p.beta != 0.0f ? load_c(p, idx) : 0.0f;
  else if constexpr (EPI == 1) return __uint_as_float(((uint32_t) static_cast<const uint16_t*>(p.aux)[idx]) << 16);
  else return static_cast<const float*>(p.aux)[idx];
}

template <int EPI>
__device__ __forceinline__ void write_new(const KParams& p, int64_t idx, float acc, float old) {
  if constexpr (EPI == 0) {
    store_c(p, idx, finish(p, acc, old));
  } else if constexpr (EPI == 1) {
    store_c(p, idx, old > 0.0f ? __fmul_rn(p.alpha, acc) : 0.0f);
  } else if constexpr (EPI == 3) {
    const float pre = finish(p, acc, old);
    if (p.aux2 != nullptr) static_cast<float*>(p.aux2)[idx] = pre;
    store_c(p, idx, lcd::gelu1(pre));
  } else if constexpr (EPI == 4) {
    store_c(p, idx, __fmul_rn(__fmul_rn(p.alpha, acc), lcd::gelu_prime1(old)));
  } else {
    const float w = __fsub_rn(old, __fmul_rn(p.lr, __fmul_rn(p.alpha, acc)));
    static_cast<float*>(const_cast<void*>(p.aux))[idx] = w;
    static_cast<uint16_t*>(p.aux2)[idx] = f32_to_bf16_rne(w);
  }
}

// Epilogue of the 32 consecutive kernel columns [n0, n0 + cnt) of one kernel row, held by one
// thread in v[]; `base` is the C index of (row, n0).  Every read goes out before the first write,
// so the loads overlap instead of queueing behind stores the compiler cannot prove disjoint.
//  * p.vec (C's columns contiguous, every row start 16-byte aligned): 16-byte loads and stores,
//    one thread covering 64 or 128 contiguous bytes per array;
//  * otherwise element by element at stride c_ns.  In the swapped skinny products C's kernel
//    rows are its columns (c_ms == 1), so the 32 lanes of a warp, which hold 32 consecutive
//    kernel rows, touch 32 consecutive elements per store.
template <int EPI>
__device__ __forceinline__ void store_row(const KParams& p, const float (&v)[32], int64_t base, int32_t cnt) {
  if (EPI < 3 && p.vec && cnt == 32) {
    if constexpr (EPI == 2) {
      float* master = static_cast<float*>(const_cast<void*>(p.aux)) + base;
      uint16_t* wb = static_cast<uint16_t*>(p.aux2) + base;
      float4 w[8];
#pragma unroll
      for (int q = 0; q < 8; q++) w[q] = *reinterpret_cast<const float4*>(master + 4 * q);
#pragma unroll
      for (int q = 0; q < 8; q++) {
        w[q].x = __fsub_rn(w[q].x, __fmul_rn(p.lr, __fmul_rn(p.alpha, v[4 * q + 0])));
        w[q].y = __fsub_rn(w[q].y, __fmul_rn(p.lr, __fmul_rn(p.alpha, v[4 * q + 1])));
        w[q].z = __fsub_rn(w[q].z, __fmul_rn(p.lr, __fmul_rn(p.alpha, v[4 * q + 2])));
        w[q].w = __fsub_rn(w[q].w, __fmul_rn(p.lr, __fmul_rn(p.alpha, v[4 * q + 3])));
        *reinterpret_cast<float4*>(master + 4 * q) = w[q];
      }
#pragma unroll
      for (int q = 0; q < 4; q++) {
        uint4 out;
        out.x = f32_to_bf16_rne(w[2 * q].x) | ((uint32_t)f32_to_bf16_rne(w[2 * q].y) << 16);
        out.y = f32_to_bf16_rne(w[2 * q].z) | ((uint32_t)f32_to_bf16_rne(w[2 * q].w) << 16);
        out.z = f32_to_bf16_rne(w[2 * q + 1].x) | ((uint32_t)f32_to_bf16_rne(w[2 * q + 1].y) << 16);
        out.w = f32_to_bf16_rne(w[2 * q + 1].z) | ((uint32_t)f32_to_bf16_rne(w[2 * q + 1].w) << 16);
        *reinterpret_cast<uint4*>(wb + 8 * q) = out;
      }
      return;
    } else {
      // values read first (C for beta, or the bf16 mask), as 32 floats
      float old[32];
      const bool reads = EPI == 1 || p.beta != 0.0f;
      if (reads) {
        if (EPI == 0 && p.c_dtype == LC_F32) {
          const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.c) + base);
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const float4 o = src[q];
            old[4 * q] = o.x;
            old[4 * q + 1] = o.y;
            old[4 * q + 2] = o.z;
            old[4 * q + 3] = o.w;
          }
        } else {
          const uint4* src = reinterpret_cast<const uint4*>(
              static_cast<const uint16_t*>(EPI == 1 ? p.aux : static_cast<const void*>(p.c)) + base);
          uint4 raw[4];
#pragma unroll
          for (int q = 0; q < 4; q++) raw[q] = src[q];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const uint32_t w4[4] = {raw[q].x, raw[q].y, raw[q].z, raw[q].w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const uint16_t lo = (uint16_t)(w4[e] & 0xffffu), hi = (uint16_t)(w4[e] >> 16);
              if (EPI == 1) {
                old[8 * q + 2 * e] = __uint_as_float((uint32_t)lo << 16);
                old[8 * q + 2 * e + 1] = __uint_as_float((uint32_t)hi << 16);
              } else {
                old[8 * q + 2 * e] = from_half_bits(p, lo);
                old[8 * q + 2 * e + 1] = from_half_bits(p, hi);
              }
            }
          }
        }
      }
      float out[32];
#pragma unroll
      for (int j = 0; j < 32; j++) {
        if constexpr (EPI == 0) out[j] = finish(p, v[j], reads ? old[j] : 0.0f);
        else out[j] = old[j] > 0.0f ? __fmul_rn(p.alpha, v[j]) : 0.0f;
      }
      if (p.c_dtype == LC_F32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.c) + base);
#pragma unroll
        for (int q = 0; q < 8; q++) dst[q] = make_float4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.c) + base);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          uint4 o;
          o.x = to_half_bits(p, out[8 * q + 0]) | ((uint32_t)to_half_bits(p, out[8 * q + 1]) << 16);
          o.y = to_half_bits(p, out[8 * q + 2]) | ((uint32_t)to_half_bits(p, out[8 * q + 3]) << 16);
          o.z = to_half_bits(p, out[8 * q + 4]) | ((uint32_t)to_half_bits(p, out[8 * q + 5]) << 16);
          o.w = to_half_bits(p, out[8 * q + 6]) | ((uint32_t)to_half_bits(p, out[8 * q + 7]) << 16);
          dst[q] = o;
        }
      }
      return;
    }
  }
  float old[32];
  const bool reads = EPI != 0 || p.beta != 0.0f;
  if (reads) {
#pragma unroll
    for (int j = 0; j < 32; j++) old[j] = j < cnt ? read_old<EPI>(p, base + (int64_t)j * p.c_ns) : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < 32; j++)
    if (j < cnt) write_new<EPI>(p, base + (int64_t)j * p.c_ns, v[j], reads ? old[j] : 0.0f);
}

// Epilogue of a 32-row x 32-column block whose rows are C's contiguous axis (c_ms == 1, the
// swapped skinny products), from a transposed shared-memory tile: column j's 32 values sit in
// `slot + j * slot_stride` with row r at position r ^ 4 (j & 7), so groups of 4 rows stay
// contiguous (16-byte reads) and neither the writes nor the reads conflict on banks.  Lane l
// handles column (8 * it + l / 4) and rows 8 * (l % 4) .. + 7: one 16-byte access per array
// for 8 consecutive 16-bit elements (two for f32).  `rows`/`cols`: valid extents.
template <int EPI>
__device__ __forceinline__ void store_cols(const KParams& p, const float* slot, int slot_stride, int64_t c_base,
                                           int32_t rows, int32_t cols) {
  static_assert(EPI != 2, "the SGD epilogue writes row-contiguous weights");
  const int lane = threadIdx.x & 31;
  const int a = lane >> 2, r0 = (lane & 3) * 8;
  const bool full_rows = r0 + 8 <= rows;
  const bool reads = EPI == 1 || p.beta != 0.0f;
  // three passes, so that no shared-memory read waits behind a global store and the global
  // reads are all in flight together: (1) the tile from shared memory, (2) what the epilogue
  // reads from C or the mask, (3) compute and store
  float v[4][8];
#pragma unroll
  for (int it = 0; it < 4; it++) {
    const int j = it * 8 + a;
    const float4 lo = *reinterpret_cast<const float4*>(slot + j * slot_stride + (r0 ^ (4 * (j & 7))));
    const float4 hi = *reinterpret_cast<const float4*>(slot + j * slot_stride + ((r0 + 4) ^ (4 * (j & 7))));
    v[it][0] = lo.x; v[it][1] = lo.y; v[it][2] = lo.z; v[it][3] = lo.w;
    v[it][4] = hi.x; v[it][5] = hi.y; v[it][6] = hi.z; v[it][7] = hi.w;
  }
  float old[4][8];
#pragma unroll
  for (int it = 0; it < 4; it++) {
    const int j = it * 8 + a;
    const int64_t idx = c_base + (int64_t)j * p.c_ns + r0;
#pragma unroll
    for (int e = 0; e < 8; e++) old[it][e] = 0.0f;
    if (!reads || j >= cols || r0 >= rows) continue;
    if (!full_rows) {
      for (int e = 0; e < 8 && r0 + e < rows; e++) old[it][e] = read_old<EPI>(p, idx + e);
    } else if (EPI == 0 && p.c_dtype == LC_F32) {
      const float4 o0 = *reinterpret_cast<const float4*>(static_cast<const float*>(p.c) + idx);
      const float4 o1 = *reinterpret_cast<const float4*>(static_cast<const float*>(p.c) + idx + 4);
      old[it][0] = o0.x; old[it][1] = o0.y; old[it][2] = o0.z; old[it][3] = o0.w;
      old[it][4] = o1.x; old[it][5] = o1.y; old[it][6] = o1.z; old[it][7] = o1.w;
    } else {
      const uint4 raw = *reinterpret_cast<const uint4*>(
          static_cast<const uint16_t*>(EPI == 1 ? p.aux : static_cast<const void*>(p.c)) + idx);
      const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const uint16_t lo = (uint16_t)(w4[e] & 0xffffu), hi = (uint16_t)(w4[e] >> 16);
        old[it][2 * e] = EPI == 1 ? __uint_as_float((uint32_t)lo << 16) : from_half_bits(p, lo);
        old[it][2 * e + 1] = EPI == 1 ? __uint_as_float((uint32_t)hi << 16) : from_half_bits(p, hi);
      }
    }
  }
#pragma unroll
  for (int it = 0; it < 4; it++) {
    const int j = it * 8 + a;
    if (j >= cols || r0 >= rows) continue;
    const int64_t idx = c_base + (int64_t)j * p.c_ns + r0;
    float out[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      if constexpr (EPI == 0) out[e] = finish(p, v[it][e], old[it][e]);
      else out[e] = old[it][e] > 0.0f ? __fmul_rn(p.alpha, v[it][e]) : 0.0f;
    }
    if (!full_rows) {
      for (int e = 0; e < 8 && r0 + e < rows; e++) store_c(p, idx + e, out[e]);
    } else if (p.c_dtype == LC_F32) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.c) + idx);
      dst[0] = make_float4(out[0], out[1], out[2], out[3]);
      dst[1] = make_float4(out[4], out[5], out[6], out[7]);
    } else {
      uint4 o;
      o.x = to_half_bits(p, out[0]) | ((uint32_t)to_half_bits(p, out[1]) << 16);
      o.y = to_half_bits(p, out[2]) | ((uint32_t)to_half_bits(p, out[3]) << 16);
      o.z = to_half_bits(p, out[4]) | ((uint32_t)to_half_bits(p, out[5]) << 16);
      o.w = to_half_bits(p, out[6]) | ((uint32_t)to_half_bits(p, out[7]) << 16);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.c) + idx) = o;
    }
  }
}

// Coalesced epilogue of a warp's 32 rows x 32 columns when C's columns are contiguous: lane l
// holds row l of the block in v[].  The block goes through the warp's shared tile (rows 36
// floats apart, so 16-byte writes and reads are conflict-free) and comes back with lane l on
// row 4i + l/8, columns 4(l%8) .. + 3: every global access covers 4 rows x 32 columns, 4 lines
// (f32) or 4 half-lines (16-bit), instead of one line per lane.  A store pattern with 32 lines
// per instruction costs the LSU about 5 cycles a line, which made row-per-lane epilogues the
// bottleneck of the fused-SGD weight gradient.  RAW: store the raw f32 values to `raw` (row
// stride `raw_ld`, the split-K partials) instead of running the epilogue at C index `base`.
template <int EPI, bool RAW>
__device__ __forceinline__ void store_tile32(const KParams& p, const float (&v)[32], float* stage, int64_t base,
                                             float* raw, int64_t raw_ld, int32_t rows) {
  const int lane = threadIdx.x & 31;
  __syncwarp();  // the previous block has been read out of the tile
  float4* mine = reinterpret_cast<float4*>(stage + lane * 36);
#pragma unroll
  for (int k = 0; k < 8; k++) mine[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  __syncwarp();
  const int rr = lane >> 3, cc = (lane & 7) * 4;
  float x[8][4];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float4 t = *reinterpret_cast<const float4*>(stage + (4 * i + rr) * 36 + cc);
    x[i][0] = t.x;
    x[i][1] = t.y;
    x[i][2] = t.z;
    x[i][3] = t.w;
  }
  if constexpr (RAW) {
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (4 * i + rr < rows)
        *reinterpret_cast<float4*>(raw + (int64_t)(4 * i + rr) * raw_ld + cc) = make_float4(x[i][0], x[i][1], x[i][2], x[i][3]);
    return;
  } else if constexpr (EPI >= 3) {
    // the GELU variants, element by element from the transposed block (lane: 4 consecutive
    // columns of rows 4i + lane / 8)
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (4 * i + rr >= rows) continue;
      const int64_t idx = base + (int64_t)(4 * i + rr) * p.c_ms + cc;
      float o[4];
      const bool reads = EPI == 4 || p.beta != 0.0f;
#pragma unroll
      for (int e = 0; e < 4; e++) o[e] = reads ? read_old<EPI>(p, idx + e) : 0.0f;
#pragma unroll
      for (int e = 0; e < 4; e++) write_new<EPI>(p, idx + e, x[i][e], o[e]);
    }
    return;
  } else {
    // the values the epilogue reads (C for beta, the mask, the master weights), all in flight together
    float o[8][4];
    const bool reads = EPI != 0 || p.beta != 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
#pragma unroll
      for (int e = 0; e < 4; e++) o[i][e] = 0.0f;
      if (!reads || 4 * i + rr >= rows) continue;
      const int64_t idx = base + (int64_t)(4 * i + rr) * p.c_ms + cc;
      if (EPI == 2) {
        // the master weights stream through once: evict-first, so that they do not push the
        // product's operands out of L2
        const float4 t = __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(p.aux) + idx));
        o[i][0] = t.x;
        o[i][1] = t.y;
        o[i][2] = t.z;
        o[i][3] = t.w;
      } else if (EPI == 0 && p.c_dtype == LC_F32) {
        const float4 t = *reinterpret_cast<const float4*>(static_cast<const float*>(p.c) + idx);
        o[i][0] = t.x;
        o[i][1] = t.y;
        o[i][2] = t.z;
        o[i][3] = t.w;
      } else {
        const uint2 t = *reinterpret_cast<const uint2*>(
            static_cast<const uint16_t*>(EPI == 1 ? p.aux : static_cast<const void*>(p.c)) + idx);
        const uint16_t h[4] = {(uint16_t)(t.x & 0xffffu), (uint16_t)(t.x >> 16), (uint16_t)(t.y & 0xffffu),
                               (uint16_t)(t.y >> 16)};
#pragma unroll
        for (int e = 0; e < 4; e++) o[i][e] = EPI == 1 ? __uint_as_float((uint32_t)h[e] << 16) : from_half_bits(p, h[e]);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (4 * i + rr >= rows) continue;
      const int64_t idx = base + (int64_t)(4 * i + rr) * p.c_ms + cc;
      float out[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        if constexpr (EPI == 0) out[e] = finish(p, x[i][e], o[i][e]);
        else if constexpr (EPI == 1) out[e] = o[i][e] > 0.0f ? __fmul_rn(p.alpha, x[i][e]) : 0.0f;
        else out[e] = __fsub_rn(o[i][e], __fmul_rn(p.lr, __fmul_rn(p.alpha, x[i][e])));
      }
      if constexpr (EPI == 2) {
        __stcs(reinterpret_cast<float4*>(static_cast<float*>(const_cast<void*>(p.aux)) + idx),
               make_float4(out[0], out[1], out[2], out[3]));
        __stcs(reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.aux2) + idx),
               make_uint2(f32_to_bf16_rne(out[0]) | ((uint32_t)f32_to_bf16_rne(out[1]) << 16),
                          f32_to_bf16_rne(out[2]) | ((uint32_t)f32_to_bf16_rne(out[3]) << 16)));
      } else if (p.c_dtype == LC_F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(p.c) + idx) = make_float4(out[0], out[1], out[2], out[3]);
      } else {
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.c) + idx) =
            make_uint2(to_half_bits(p, out[0]) | ((uint32_t)to_half_bits(p, out[1]) << 16),
                       to_half_bits(p, out[2]) | ((uint32_t)to_half_bits(p, out[3]) << 16));
      }
    }
  }
}

// Fused-SGD epilogue, software-pipelined over the 32-column groups of a row block: the master
// weights of group g + 1 are loaded (into `next`) before group g is computed, so their load
// latency overlaps a whole group's TMEM read, transpose and stores instead of stalling every
// group (measured: 2.3 us per group with the loads issued in-line).  Lane layout as in
// store_tile32: lane = 8 * (row % 4) + column quad, rows 4 i + lane / 8.
__device__ __forceinline__ void load_master_block(const KParams& p, int64_t base, int32_t rows, float (&o)[8][4]) {
  const int lane = threadIdx.x & 31;
  const int rr = lane >> 3, cc = (lane & 7) * 4;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    if (4 * i + rr < rows)
      t = __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(p.aux) + base + (int64_t)(4 * i + rr) * p.c_ms + cc));
    o[i][0] = t.x;
    o[i][1] = t.y;
    o[i][2] = t.z;
    o[i][3] = t.w;
  }
}

__device__ __forceinline__ void sgd_block32(const KParams& p, const uint32_t (&r)[32], float* stage, int64_t base,
                                            int32_t rows, const float (&o)[8][4]) {
  const int lane = threadIdx.x & 31;
  __syncwarp();  // the previous block has been read out of the tile
  float4* mine = reinterpret_cast<float4*>(stage + lane * 36);
#pragma unroll
  for (int k = 0; k < 8; k++)
    mine[k] = make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]), __uint_as_float(r[4 * k + 2]),
                          __uint_as_float(r[4 * k + 3]));
  __syncwarp();
  const int rr = lane >> 3, cc = (lane & 7) * 4;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if (4 * i + rr >= rows) continue;
    const float4 t = *reinterpret_cast<const float4*>(stage + (4 * i + rr) * 36 + cc);
    const float x[4] = {t.x, t.y, t.z, t.w};
    float out[4];
#pragma unroll
    for (int e = 0; e < 4; e++) out[e] = __fsub_rn(o[i][e], __fmul_rn(p.lr, __fmul_rn(p.alpha, x[e])));
    const int64_t idx = base + (int64_t)(4 * i + rr) * p.c_ms + cc;
    __stcs(reinterpret_cast<float4*>(static_cast<float*>(const_cast<void*>(p.aux)) + idx),
           make_float4(out[0], out[1], out[2], out[3]));
    __stcs(reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.aux2) + idx),
           make_uint2(f32_to_bf16_rne(out[0]) | ((uint32_t)f32_to_bf16_rne(out[1]) << 16),
                      f32_to_bf16_rne(out[2]) | ((uint32_t)f32_to_bf16_rne(out[3]) << 16)));
  }
}

__device__ __forceinline__ float* partial_row(const KParams& p, int32_t split, int32_t b, int32_t m) {
  return p.partial + (((int64_t)split * p.batch + b) * p.M + m) * (int64_t)p.N;
}

// Raw split-K partial of 32 columns of one row: 128 contiguous bytes per thread when they fit.
__device__ __forceinline__ void store_partial(const KParams& p, const float (&v)[32], float* dst, int32_t cnt) {
  if (cnt == 32 && (p.N % 4) == 0) {
#pragma unroll
    for (int q = 0; q < 8; q++)
      reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++)
      if (j < cnt) dst[j] = v[j];
  }
}

// Sum of the splits' partials of 32 columns of one row, in split order from +0 (for up to 8
// splits the separate reduce kernel's order is this one too).
__device__ __forceinline__ void sum_partials(const KParams& p, float (&v)[32], int32_t b, int32_t m, int32_t n0,
                                             int32_t cnt) {
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = 0.0f;
  if (cnt == 32 && (p.N % 4) == 0) {
    for (int s = 0; s < p.splits; s++) {
      const float4* src = reinterpret_cast<const float4*>(partial_row(p, s, b, m) + n0);
      float4 t[8];
#pragma unroll
      for (int q = 0; q < 8; q++) t[q] = __ldcg(src + q);
#pragma unroll
      for (int q = 0; q < 8; q++) {
        v[4 * q + 0] = __fadd_rn(v[4 * q + 0], t[q].x);
        v[4 * q + 1] = __fadd_rn(v[4 * q + 1], t[q].y);
        v[4 * q + 2] = __fadd_rn(v[4 * q + 2], t[q].z);
        v[4 * q + 3] = __fadd_rn(v[4 * q + 3], t[q].w);
      }
    }
  } else {
    for (int s = 0; s < p.splits; s++) {
      const float* src = partial_row(p, s, b, m) + n0;
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (j < cnt) v[j] = __fadd_rn(v[j], __ldcg(src + j));
    }
  }
}

// 32 columns [n0, n0 + 32) of row m of one batch's product over K values [k0, k1), summed in k
// order from +0 with separately rounded products (IEEE infinities and NaNs as the CPU backend
// gives them), written to out[0..31]: the 3xTF32 path's fallback for units whose operands are
// not all finite.  One column at a time, so it holds few registers in the epilogue warps.
__device__ __noinline__ void exact_f32_row(const float* fa, const float* fb, int64_t fa_ms, int64_t fa_ks,
                                           int64_t fa_bs, int64_t fb_ns, int64_t fb_ks, int64_t fb_bs, int32_t M,
                                           int32_t N, int32_t b, int32_t m, int32_t n0, int64_t k0, int64_t k1,
                                           float* out) {
  const float* arow = fa + (int64_t)b * fa_bs + (int64_t)m * fa_ms;
  for (int j = 0; j < 32; j++) {
    float acc = 0.0f;
    if (m < M && n0 + j < N) {
      const float* bcol = fb + (int64_t)b * fb_bs + (int64_t)(n0 + j) * fb_ns;
      for (int64_t k = k0; k < k1; k++) acc = __fadd_rn(acc, __fmul_rn(arow[k * fa_ks], bcol[k * fb_ks]));
    }
    out[j] = acc;
  }
}

// ---- where a kernel's products come from ------------------------------------------------------
// OneProduct: the tensor maps and parameters of a single product, passed as kernel arguments.
// ChainParams/ChainSrc: a chain of dependent products in one launch (product l + 1 reads what
// product l writes), for the pipeline's per-microbatch layer loops; CTAs stay resident across
// the chain and meet at a counter per product instead of a kernel boundary.
struct OneProduct {
  const CUtensorMap* a;
  const CUtensorMap* b;
  const KParams* p;
  __device__ __forceinline__ int layers() const { return 1; }
  __device__ __forceinline__ const KParams& kp(int) const { return *p; }
  __device__ __forceinline__ const CUtensorMap* map_a(int) const { return a; }
  __device__ __forceinline__ const CUtensorMap* map_b(int) const { return b; }
  __device__ __forceinline__ int* counters() const { return nullptr; }
  __device__ __forceinline__ bool a_stable() const { return false; }
};

constexpr int kMaxChain = 32;

struct ChainParams {
  CUtensorMap a[kMaxChain];
  CUtensorMap b[kMaxChain];
  KParams p[kMaxChain];
  int32_t n;
  int32_t a_stable;  // no kernel that may still be running writes any A operand (the weights)
  int* counters;     // [n], zero at launch: CTAs whose epilogue finished product l
};

struct ChainSrc {
  const ChainParams* cp;
  __device__ __forceinline__ int layers() const { return cp->n; }
  // by value: read once per product, not re-read from the parameter block inside the loops
  __device__ __forceinline__ KParams kp(int l) const { return cp->p[l]; }
  __device__ __forceinline__ const CUtensorMap* map_a(int l) const { return &cp->a[l]; }
  __device__ __forceinline__ const CUtensorMap* map_b(int l) const { return &cp->b[l]; }
  __device__ __forceinline__ int* counters() const { return cp->counters; }
  __device__ __forceinline__ bool a_stable() const { return cp->a_stable != 0; }
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *counter >= target (every CTA's epilogue finished the previous product),
// then orders those generic-proxy writes before this thread's TMA (async-proxy) reads.
__device__ __forceinline__ bool wait_counter(const int* counter, int target, int* err) {
  const uint64_t t0 = lcd::global_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_gpu(counter) >= target) break;
    __nanosleep(32);  // 128 pollers of one line: leave the L2 some room for the arrivals
    if ((i & 63u) == 63u) {
      if (*(volatile int*)err != 0) return false;
      if (lcd::global_ns() - t0 > lcd::kWaitLimitNs) {
        atomicOr(err, 1);
        return false;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// TWO_SM: the 256-row tile of a unit is computed by a pair of CTAs with cta_group::2 MMAs
// (rows 128 * (rank & 1) .. + 127 of the tile live in that CTA's TMEM, the even CTA issues the
// MMAs); a unit is one output tile and
// the pair walks the units together.
template <int BN, bool TF32X3, int EPI, bool PAIR, class Src, bool TWO_SM = false>
__device__ __forceinline__ void gemm_body(const Src& src) {
  using C = Cfg<BN, TF32X3, PAIR, TWO_SM>;
  int* const err = src.kp(0).err;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // ring layout: [A hi][B hi] per stage, then (3xTF32) [A lo][B lo] per stage
  auto a_hi = [&](int s) { return smem + s * (C::A_BYTES + C::B_BYTES); };
  auto b_hi = [&](int s) { return smem + s * (C::A_BYTES + C::B_BYTES) + C::A_BYTES; };
  uint8_t* lo_base = smem + C::STAGES * (C::A_BYTES + C::B_BYTES);
  auto a_lo = [&](int s) { return lo_base + s * (C::A_BYTES + C::B_BYTES); };
  auto b_lo = [&](int s) { return lo_base + s * (C::A_BYTES + C::B_BYTES) + C::A_BYTES; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* conv = bars + 2 * C::STAGES;
  uint64_t* tfull = bars + 3 * C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* recv_full = drain + 1;  // PAIR: the peer's half-tile has landed here (128 arrivals)
  uint64_t* recv_free = drain + 2;  // PAIR: the peer has consumed what this CTA sent it (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 3);
  uint32_t* layer_done = tmem_slot + 1;  // chain: epilogue warps done with their products so far
  // 3xTF32: stamp uo + 1 in slot uo & 7 when the converters of this CTA's unit ordinal uo meet an
  // infinity or NaN (the converters run at most a few units ahead of the epilogue)
  uint32_t* nonfinite = layer_done + 1;
  float* recv = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + ((C::BAR_BYTES + 15) / 16) * 16);
  float* epi_stage = recv + C::RECV_BYTES / 4;  // non-pair kernels: 4 x (32 x 36) f32

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      lcd::mbar_init(&full[s], 1);
      lcd::mbar_init(&empty[s], 1);
      lcd::mbar_init(&conv[s], C::CONV_THREADS);
    }
    for (int a = 0; a < 2; a++) {
      lcd::mbar_init(&tfull[a], 1);
      // one arrival per epilogue warp (2-SM: both CTAs' warps, on the leader)
      lcd::mbar_init(&tempty[a], TWO_SM ? 8 : 4);
    }
    lcd::mbar_init(drain, 1);
    lcd::mbar_init(recv_full, 128);
    lcd::mbar_init(recv_free, 128);
    *layer_done = 0;
    for (int i = 0; i < 8; i++) nonfinite[i] = 0;
    lcd::fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (TWO_SM) {
      lcd::tmem_alloc_2sm(tmem_slot, C::TMEM_COLS);
      lcd::tmem_relinquish_2sm();
    } else {
      lcd::tmem_alloc(tmem_slot, C::TMEM_COLS);
      lcd::tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    for (int l = 0; l < src.layers(); l++) {
      lcd::tma_prefetch_desc(src.map_a(l));
      lcd::tma_prefetch_desc(src.map_b(l));
    }
  }
  lcd::tc_fence_before();
  __syncthreads();
  lcd::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // both CTAs of a pair have initialised their barriers before either arrives on the other's
  if constexpr (PAIR || TWO_SM) lcd::cluster_sync();
  const uint32_t rank = (PAIR || TWO_SM) ? lcd::cluster_ctarank() : 0u;
  // QUAD (PAIR and TWO_SM): a cluster of 4 is two 2-SM pairs, pair kh = rank >> 1 computing K
  // half kh of the same 256-row tile; the pairs exchange partials as PAIR CTAs do.
  constexpr bool QUAD = PAIR && TWO_SM;
  const uint32_t leader = rank & ~1u;                    // the even CTA of this CTA's 2-SM pair
  const bool is_leader = !TWO_SM || (rank & 1u) == 0u;  // issues the MMAs and arms the stages
  const uint32_t kh = QUAD ? rank >> 1 : rank;           // PAIR: the K half this CTA (pair) sums
  // the units this CTA walks: every CTA on its own, (TWO_SM) the pair together, or (QUAD) the pair
  // with the other pair of its cluster on the other split of the same tile
  const int32_t u_first = QUAD     ? (int32_t)(((blockIdx.x >> 2) << 1) | (rank >> 1))
                          : TWO_SM ? (int32_t)(blockIdx.x >> 1)
                                   : (int32_t)blockIdx.x;
  const int32_t u_step = QUAD ? (int32_t)((gridDim.x >> 2) << 1) : TWO_SM ? (int32_t)(gridDim.x >> 1) : (int32_t)gridDim.x;
  // first C row of a unit's tile row tm held by this CTA
  auto tile_row0 = [&](int32_t tm) -> int32_t { return TWO_SM ? tm * 256 + (int32_t)(rank & 1u) * 128 : tm * kBM; };
  // Programmatic dependent launch: the next kernel on the stream may start its own set-up now.
  // Everything below that reads or writes global memory first waits for the previous kernel.
  lcd::griddep_launch_dependents();

  // bytes one stage's full barrier waits for (TWO_SM: both CTAs' loads land on the leader's)
  constexpr uint32_t kStageTx = (C::A_BYTES + C::B_BYTES) * (TWO_SM ? 2 : 1);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      // Each product's loads are gated on what produced its inputs: the previous kernel for the
      // first product (programmatic dependent launch), the previous product's counter inside a
      // chain.  When the A operands are stable (weights nobody is writing), A is loaded ahead of
      // the gate into up to STAGES slots and only the B loads wait.
      const uint64_t once = lcd::policy_evict_first();
      const uint64_t keep = lcd::policy_evict_last();
      const uint64_t normal = lcd::policy_evict_normal();
      int s = 0;
      uint32_t ph = 0;
      uint32_t filled = 0, last_par = 0;  // bit s: stage s filled at least once / parity of its last fill
      bool ok = true;
      for (int l = 0; ok && l < src.layers(); l++) {
        decltype(auto) p = src.kp(l);  // a chain's are copied to registers once per product
        const CUtensorMap* ta = src.map_a(l);
        const CUtensorMap* tb = src.map_b(l);
        auto gate = [&]() -> bool {
          if (l == 0) {
            lcd::griddep_wait();
            return true;
          }
          return wait_counter(src.counters() + (l - 1), (int)gridDim.x, err);
        };
        bool open = !src.a_stable();
        if (open && !gate()) {
          ok = false;
          break;
        }
        // B loads held back until the gate opens: (stage, k0, tn, b)
        int32_t pend[C::STAGES][4];
        int npend = 0;
        auto load = [&](int st, void* dst, const CUtensorMap* map, int32_t c0, int32_t c1, int32_t b, bool hint) {
          if constexpr (TWO_SM) {
            // bytes count on the leader's barrier for this stage
            lcd::tma_load_3d_2sm(dst, map, lcd::rank_addr(lcd::smem_u32(&full[st]), leader), c0, c1, b,
                                 hint ? once : (EPI == 2 ? keep : normal));
          } else {
            if (hint) lcd::tma_load_3d_hint(dst, map, &full[st], c0, c1, b, once);
            else if (EPI == 2) lcd::tma_load_3d_hint(dst, map, &full[st], c0, c1, b, keep);
            else lcd::tma_load_3d(dst, map, &full[st], c0, c1, b);
          }
        };
        // this CTA's rows of the B^T tile: all BN, or (TWO_SM) its half
        constexpr int kBRows = TWO_SM ? BN / 2 : BN;
        const int32_t b_row_off = TWO_SM ? (int32_t)(rank & 1u) * kBRows : 0;
        auto load_b = [&](int st, int32_t k0, int32_t tn, int32_t b) {
          if (!p.b_mn) {
            load(st, b_hi(st), tb, k0, tn * BN + b_row_off, b, p.b_once);
          } else {
#pragma unroll
            for (int j = 0; j < kBRows / C::EPR; j++)
              load(st, b_hi(st) + j * (C::BK * kRowBytes), tb, tn * BN + b_row_off + j * C::EPR, k0, b, p.b_once);
          }
        };
        auto release = [&]() -> bool {
          if (!gate()) return false;
          for (int i = 0; i < npend; i++) load_b(pend[i][0], pend[i][1], pend[i][2], pend[i][3]);
          npend = 0;
          open = true;
          return true;
        };
        for (int32_t u = u_first; ok && u < p.units; u += u_step) {
          int32_t b, split, tm, tn;
          unit_coords(p, u, &b, &split, &tm, &tn);
          const int32_t kb = split * p.kt_per_split;
          const int32_t ke = min(kb + p.kt_per_split, p.k_tiles);
          const int32_t a_row0 = tile_row0(tm);
          // The streamed operand's DRAM reads run `prefetch` k-tiles ahead through L2, beyond the
          // few the shared-memory ring holds; its ring loads then find the tiles in L2.
          auto prefetch_a = [&](int32_t kt) {
            if (!p.a_mn) {
              lcd::tma_prefetch_l2_3d(ta, kt * C::BK, a_row0, b);
            } else {
#pragma unroll
              for (int j = 0; j < kBM / C::EPR; j++) lcd::tma_prefetch_l2_3d(ta, a_row0 + j * C::EPR, kt * C::BK, b);
            }
          };
          if (p.prefetch > 0 && p.a_once)
            for (int32_t kt = kb + C::STAGES; kt < min(ke, kb + p.prefetch); kt++) prefetch_a(kt);
          for (int32_t kt = kb; kt < ke; kt++) {
            if (p.prefetch > 0 && p.a_once && kt + p.prefetch < ke) prefetch_a(kt + p.prefetch);
            // every slot holds an A tile waiting for its B: open the gate before reusing one
            if (!open && npend == C::STAGES && !release()) {
              ok = false;
              break;
            }
            if (!lcd::mbar_wait(&empty[s], ph ^ 1u, err)) {
              ok = false;
              break;
            }
            // TWO_SM: only the leader arms the stage (with both CTAs' bytes); the peer's loads
            // may land first, which an mbarrier allows while its arrival is still pending
            if (is_leader) lcd::mbar_arrive_expect_tx(&full[s], kStageTx);
            const int32_t k0 = kt * C::BK;
            if (!p.a_mn) {
              load(s, a_hi(s), ta, k0, a_row0, b, p.a_once);
            } else {
#pragma unroll
              for (int j = 0; j < kBM / C::EPR; j++)
                load(s, a_hi(s) + j * (C::BK * kRowBytes), ta, a_row0 + j * C::EPR, k0, b, p.a_once);
            }
            if (open) {
              load_b(s, k0, tn, b);
            } else {
              pend[npend][0] = s;
              pend[npend][1] = k0;
              pend[npend][2] = tn;
              pend[npend][3] = b;
              npend++;
            }
            filled |= 1u << s;
            last_par = (last_par & ~(1u << s)) | (ph << s);
            if (++s == C::STAGES) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
        // a product with fewer k-tiles than stages (or none for this CTA) still opens its gate
        if (ok && !open && !release()) ok = false;
      }
      // never leave a bulk copy in flight into shared memory that is about to be released (the
      // 2-SM peer's copies complete on the leader's barriers; the closing cluster barrier covers
      // them, as the leader waits here first)
      if (is_leader)
        for (int t = 0; t < C::STAGES; t++)
          if (filled & (1u << t)) lcd::mbar_wait(&full[t], (last_par >> t) & 1u, err);
    }
  } else if (warp == 1) {
    if (lane == 0 && is_leader) {
      // ---------------- MMA issuer (TWO_SM: the leader, for both CTAs) ----------------
      // The accumulator is handed to the epilogue every KC k-tiles (a "chunk"): once per unit for
      // 16-bit inputs, every kChunkTiles k-tiles for 3xTF32, whose long sums the epilogue then
      // adds with round-to-nearest (the tensor core's own f32 accumulation truncates).
      int s = 0;
      uint32_t ph = 0;
      int32_t h = 0;  // hand-offs so far
      bool ok = true;
      for (int l = 0; ok && l < src.layers(); l++) {
      decltype(auto) p = src.kp(l);  // a chain's are copied to registers once per product
      for (int32_t u = u_first; ok && u < p.units; u += u_step) {
        int32_t b, split, tm, tn;
        unit_coords(p, u, &b, &split, &tm, &tn);
        (void)b;
        (void)tm;
        (void)tn;
        const int32_t kb = split * p.kt_per_split;
        const int32_t ke = min(kb + p.kt_per_split, p.k_tiles);
        for (int32_t c0 = kb; ok && c0 < ke; c0 += C::KC, h++) {
        const int32_t c1 = min(c0 + C::KC, ke);
        const int acc = h & 1;
        if (!lcd::mbar_wait(&tempty[acc], ((h >> 1) & 1) ^ 1u, err)) {
          ok = false;
          break;
        }
        lcd::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int32_t kt = c0; kt < c1; kt++) {
          if (!lcd::mbar_wait(TF32X3 ? &conv[s] : &full[s], ph, err)) {
            ok = false;
            break;
          }
          lcd::tc_fence_after();
          const uint32_t sa = lcd::smem_u32(a_hi(s)), sb = lcd::smem_u32(b_hi(s));
          const uint32_t sal = lcd::smem_u32(a_lo(s)), sbl = lcd::smem_u32(b_lo(s));
          // K-major: 8-row x 128-byte swizzle atoms stacked along MN (SBO 1024), the k-step moves
          // 32 bytes inside the atom.  MN-major: 128-byte rows along MN, chunks of EPR columns
          // BK rows apart (LBO); the k-step moves UMMA_K rows.  32-bit MN-major tiles use the
          // 32-byte-atom swizzle, whose atoms are 4 rows (SBO 512).
          constexpr uint32_t mn_layout = TF32X3 ? lcd::kLayoutSw128Atom32 : lcd::kLayoutSw128;
          constexpr uint32_t mn_sbo = TF32X3 ? 512u : 1024u;
          const uint32_t a_lay = p.a_mn ? mn_layout : lcd::kLayoutSw128;
          const uint32_t b_lay = p.b_mn ? mn_layout : lcd::kLayoutSw128;
          const uint32_t a_lbo = p.a_mn ? C::BK * kRowBytes : 16;
          const uint32_t b_lbo = p.b_mn ? C::BK * kRowBytes : 16;
          const uint32_t a_sbo = p.a_mn ? mn_sbo : 1024u;
          const uint32_t b_sbo = p.b_mn ? mn_sbo : 1024u;
#pragma unroll
          for (int ks = 0; ks < C::KSTEPS; ks++) {
            const uint32_t a_off = p.a_mn ? ks * C::UMMA_K * kRowBytes : ks * 32;
            const uint32_t b_off = p.b_mn ? ks * C::UMMA_K * kRowBytes : ks * 32;
            const uint64_t da = lcd::smem_desc(sa + a_off, a_lbo, a_sbo, a_lay);
            const uint64_t db = lcd::smem_desc(sb + b_off, b_lbo, b_sbo, b_lay);
            const uint32_t accum = (kt > c0 || ks > 0) ? 1u : 0u;
            if constexpr (TF32X3) {
              const uint64_t dal = lcd::smem_desc(sal + a_off, a_lbo, a_sbo, a_lay);
              const uint64_t dbl = lcd::smem_desc(sbl + b_off, b_lbo, b_sbo, b_lay);
              lcd::umma_tf32(d_tmem, dal, db, p.idesc, accum);  // lo(A) * hi(B)
              lcd::umma_tf32(d_tmem, da, dbl, p.idesc, 1u);     // hi(A) * lo(B)
              lcd::umma_tf32(d_tmem, da, db, p.idesc, 1u);      // hi(A) * hi(B)
            } else if constexpr (TWO_SM) {
              lcd::umma_f16_2sm(d_tmem, da, db, p.idesc, accum);
            } else {
              lcd::umma_f16(d_tmem, da, db, p.idesc, accum);
            }
          }
          if constexpr (TWO_SM) lcd::umma_commit_2sm_pair(&empty[s], leader);  // frees the stage in both CTAs
          else lcd::umma_commit(&empty[s]);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (TWO_SM) lcd::umma_commit_2sm_pair(&tfull[acc], leader);
        else lcd::umma_commit(&tfull[acc]);
        }
      }
      }
      // every MMA this thread issued has retired before TMEM is released
      if constexpr (TWO_SM) lcd::umma_commit_2sm(drain);
      else lcd::umma_commit(drain);
      lcd::mbar_wait(drain, 0, err);
    }
  } else if (warp < 6) {
    // ---------------- epilogue ----------------
    // Warp q owns TMEM lanes (tile rows) 32q..32q+31; lane l holds tile row 32q + l.
    const int q = warp & 3;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    int32_t h = 0;
    bool ok = true;
    uint32_t uo = 0;  // unit ordinal (the converters count the same units)
    uint32_t xr = 0;  // PAIR: exchange rounds so far (the receive barriers' phase)
    lcd::griddep_wait();
    for (int l = 0; ok && l < src.layers(); l++) {
    decltype(auto) p = src.kp(l);  // a chain's are copied to registers once per product
    const bool split_mode = p.splits > 1 && !PAIR;
    for (int32_t u = u_first; ok && u < p.units; u += u_step, uo++) {
      int32_t b, split, tm, tn;
      unit_coords(p, u, &b, &split, &tm, &tn);
      const int32_t m = tile_row0(tm) + q * 32 + lane;
      const int64_t c_row = p.c_off + (int64_t)b * p.c_bs + (int64_t)m * p.c_ms;
      // one 32-column group [n0, n0 + 32) of this lane's row, straight from the tcgen05.ld registers
      // (warp-uniform branches: n0, cnt and the block's row count are the same for all lanes)
      auto emit = [&](const uint32_t (&r)[32], int32_t n0) {
        const int32_t cnt = min(32, p.N - n0);
        const int32_t m0w = tile_row0(tm) + q * 32;
        const int32_t rows = min(32, p.M - m0w);
        if (cnt <= 0 || rows <= 0) return;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
        float* stage = epi_stage + (warp - 2) * (32 * 36);
        if (split_mode) {
          if (!PAIR && cnt == 32 && (p.N % 4) == 0)
            store_tile32<EPI, true>(p, v, stage, 0, partial_row(p, split, b, m0w) + n0, p.N, rows);
          else if (m < p.M)
            store_partial(p, v, partial_row(p, split, b, m) + n0, cnt);
        } else if (!PAIR && p.vec && cnt == 32) {
          store_tile32<EPI, false>(p, v, stage, p.c_off + (int64_t)b * p.c_bs + (int64_t)m0w * p.c_ms + n0, nullptr,
                                   0, rows);
        } else if (m < p.M) {
          store_row<EPI>(p, v, c_row + (int64_t)n0 * p.c_ns, cnt);
        }
      };
      if constexpr (TF32X3) {
        // Running sum of the chunk accumulators, kept in a third TMEM region (columns 2*BN..3*BN)
        // and updated with round-to-nearest f32 adds.
        const int32_t kb = split * p.kt_per_split;
        const int32_t ke = min(kb + p.kt_per_split, p.k_tiles);
        const uint32_t run_base = lane_base + 2 * BN;
        bool first = true;
        for (int32_t c0 = kb; c0 < ke; c0 += C::KC, h++) {
          const int acc = h & 1;
          if (!lcd::mbar_wait(&tfull[acc], (h >> 1) & 1, p.err)) {
            ok = false;
            break;
          }
          lcd::tc_fence_after();
#pragma unroll 1
          for (int g = 0; g < BN / 32; g++) {
            uint32_t r[32];
            lcd::tmem_ld_32x32b_x32(lane_base + acc * BN + g * 32, r);
            lcd::tmem_ld_wait();
            if (!first) {
              uint32_t o[32];
              lcd::tmem_ld_32x32b_x32(run_base + g * 32, o);
              lcd::tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; j++) r[j] = __float_as_uint(__fadd_rn(__uint_as_float(o[j]), __uint_as_float(r[j])));
            }
            lcd::tmem_st_32x32b_x32(run_base + g * 32, r);
            lcd::tmem_st_wait();
          }
          first = false;
          lcd::tc_fence_before();
          __syncwarp();
          if (lane == 0) lcd::mbar_arrive(&tempty[acc]);
        }
        if (!ok) break;
        // every conversion of this unit preceded its last hand-off, so its stamp is in place
        const bool exact = *reinterpret_cast<volatile uint32_t*>(&nonfinite[uo & 7]) == uo + 1;
#pragma unroll 1
        for (int g = 0; g < BN / 32; g++) {
          uint32_t r[32];
          if (!exact) {
            lcd::tmem_ld_32x32b_x32(run_base + g * 32, r);
            lcd::tmem_ld_wait();
          } else {
            // through this warp's staging tile (row = lane), read back before emit reuses it
            float* row = epi_stage + (warp - 2) * (32 * 36) + lane * 36;
            exact_f32_row(p.fa, p.fb, p.fa_ms, p.fa_ks, p.fa_bs, p.fb_ns, p.fb_ks, p.fb_bs, p.M, p.N, b, m,
                          tn * BN + g * 32, (int64_t)kb * C::BK, min((int64_t)ke * C::BK, p.K), row);
#pragma unroll
            for (int j = 0; j < 32; j++) r[j] = __float_as_uint(row[j]);
            __syncwarp();
          }
          emit(r, tn * BN + g * 32);
        }
      } else if constexpr (PAIR) {
        // CTA pair (cluster of 2) splitting K in halves.  Rank r finalises the column half r of
        // the tile: each CTA writes the raw accumulator columns of the other half into the
        // other's receive buffer through distributed shared memory, then adds what it received
        // to its own half in split order (rank 0's partial first, from +0, as the global split-K
        // paths sum) and runs the epilogue.  The half goes over in EXCH_ROUNDS rounds of
        // RECV_COLS columns (one round up to BN = 128).  Receive buffer: 128 rows x RECV_COLS
        // floats, 16-byte chunk c of row r stored at c ^ (r & 7), so the 32 rows a warp touches
        // at once spread over all banks.
        constexpr int HB = C::RECV_COLS;  // floats per receive-buffer row
        constexpr int GR = HB / 32;       // 32-column groups per round
        constexpr int GH = BN / 64;       // 32-column groups per half
        const int acc = h & 1;
        if (!lcd::mbar_wait(&tfull[acc], (h >> 1) & 1, p.err)) {
          ok = false;
          break;
        }
        lcd::tc_fence_after();
        const int row = q * 32 + lane;
        const uint32_t sw = (uint32_t)(row & 7);
        const uint32_t peer = QUAD ? rank ^ 2u : rank ^ 1u;  // the CTA with the other K half of these rows
#pragma unroll 1
        for (int rd = 0; ok && rd < C::EXCH_ROUNDS; rd++, xr++) {
        // (1) this round's columns of the peer's half, once the peer has consumed what this CTA
        // sent it last round
        if (!lcd::mbar_wait_cluster(recv_free, (xr & 1) ^ 1, p.err)) {
          ok = false;
          break;
        }
        {
          const uint32_t dst = lcd::mapa_shared(lcd::smem_u32(recv + row * HB), peer);
          uint32_t r[GR][32];
#pragma unroll
          for (int gl = 0; gl < GR; gl++)
            lcd::tmem_ld_32x32b_x32(lane_base + acc * BN + ((kh ^ 1u) * GH + rd * GR + gl) * 32, r[gl]);
          lcd::tmem_ld_wait();
#pragma unroll
          for (int gl = 0; gl < GR; gl++) {
#pragma unroll
            for (int k = 0; k < 8; k++) {
              const uint32_t chunk = (uint32_t)(gl * 8) + ((uint32_t)k ^ sw);
              lcd::st_cluster_v4(dst + chunk * 16, __uint_as_float(r[gl][4 * k]), __uint_as_float(r[gl][4 * k + 1]),
                                 __uint_as_float(r[gl][4 * k + 2]), __uint_as_float(r[gl][4 * k + 3]));
            }
          }
        }
        lcd::mbar_arrive_remote(lcd::mapa_shared(lcd::smem_u32(recv_full), peer));
        // (2) the same columns of this CTA's half: its own accumulator plus the peer's, then the
        // epilogue
        if (!lcd::mbar_wait_cluster(recv_full, xr & 1, p.err)) {
          ok = false;
          break;
        }
        const float* src = recv + row * HB;
#pragma unroll 1
        for (int gl = 0; gl < GR; gl++) {
          const int g = (int)kh * GH + rd * GR + gl;
          uint32_t r[32];
          lcd::tmem_ld_32x32b_x32(lane_base + acc * BN + g * 32, r);
          lcd::tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const uint32_t chunk = (uint32_t)(gl * 8) + ((uint32_t)k ^ sw);
            const float4 o = *reinterpret_cast<const float4*>(src + chunk * 4);
            const float in[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float mine = __uint_as_float(r[4 * k + e]);
              v[4 * k + e] = kh == 0 ? __fadd_rn(__fadd_rn(0.0f, mine), in[e]) : __fadd_rn(__fadd_rn(0.0f, in[e]), mine);
            }
          }
          const int32_t n0 = tn * BN + g * 32;
          const int32_t cnt = min(32, p.N - n0);
          if (p.tvec) {
            // transpose through this warp's rows of the receive buffer (group gl's 128 bytes of
            // each row, read above by every lane: hence the first __syncwarp): column j's 32
            // values go to row j of the area, row r at position r ^ 4 (j & 7)
            float* slot = recv + (q * 32) * HB + gl * 32;
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; j++) slot[j * HB + (lane ^ (4 * (j & 7)))] = v[j];
            __syncwarp();
            const int32_t mw = tile_row0(tm) + q * 32;
            store_cols<EPI>(p, slot, HB, p.c_off + (int64_t)b * p.c_bs + mw + (int64_t)n0 * p.c_ns,
                            min(32, p.M - mw), cnt);
          } else if (m < p.M && cnt > 0) {
            store_row<EPI>(p, v, c_row + (int64_t)n0 * p.c_ns, cnt);
          }
        }
        lcd::mbar_arrive_remote(lcd::mapa_shared(lcd::smem_u32(recv_free), peer));
        }
        if (!ok) break;
        lcd::tc_fence_before();
        __syncwarp();
        // QUAD: the pair's leader refills both CTAs' accumulators, so both release on its barrier
        if (lane == 0) {
          if (!is_leader) lcd::mbar_arrive_remote(lcd::rank_addr(lcd::smem_u32(&tempty[acc]), leader));
          else lcd::mbar_arrive(&tempty[acc]);
        }
        h++;
      } else {
        const int acc = h & 1;
        // fused SGD over whole 32-column groups: the first group's master weights do not depend
        // on the accumulator, so they are loaded while the MMAs finish
        const int32_t m0w = tile_row0(tm) + q * 32;
        const int32_t rows = min(32, p.M - m0w);
        const bool sgd_pipe = EPI == 2 && !split_mode && p.vec && tn * BN + BN <= p.N && rows > 0;
        const int64_t base0 = p.c_off + (int64_t)b * p.c_bs + (int64_t)m0w * p.c_ms + tn * BN;
        float next[8][4];
        if (sgd_pipe) load_master_block(p, base0, rows, next);
        if (!lcd::mbar_wait(&tfull[acc], (h >> 1) & 1, p.err)) {
          ok = false;
          break;
        }
        lcd::tc_fence_after();
        // The epilogue's reads (master weights, mask, old C) wait on HBM group after group; pull
        // the next unit's rows into L2 now, a tile ahead, so that they come from L2 then.
        if (!split_mode && p.vec && ((EPI != 0 && EPI != 3) || p.beta != 0.0f) && u + u_step < p.units) {
          int32_t b2, s2, tm2, tn2;
          unit_coords(p, u + u_step, &b2, &s2, &tm2, &tn2);
          const int32_t m2 = tile_row0(tm2) + q * 32 + lane;
          const int32_t n2 = tn2 * BN;
          if (m2 < p.M && n2 < p.N) {
            const int es = (EPI == 2 || EPI == 4 || p.c_dtype == LC_F32) ? 4 : 2;
            const char* src = static_cast<const char*>((EPI == 0 || EPI == 3) ? static_cast<const void*>(p.c) : p.aux) +
                              (p.c_off + (int64_t)b2 * p.c_bs + (int64_t)m2 * p.c_ms + n2) * es;
            const int32_t bytes = min(BN, p.N - n2) * es;
            for (int32_t off = 0; off < bytes; off += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(src + off));
          }
        }
        if (sgd_pipe) {
          float* stage = epi_stage + (warp - 2) * (32 * 36);
          float o[8][4];
#pragma unroll 1
          for (int g = 0; g < BN / 32; g++) {
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
              for (int e = 0; e < 4; e++) o[i][e] = next[i][e];
            if (g + 1 < BN / 32) load_master_block(p, base0 + (g + 1) * 32, rows, next);
            uint32_t r[32];
            lcd::tmem_ld_32x32b_x32(lane_base + acc * BN + g * 32, r);
            lcd::tmem_ld_wait();
            sgd_block32(p, r, stage, base0 + g * 32, rows, o);
          }
        } else {
#pragma unroll 1
          for (int g = 0; g < BN / 32; g++) {
            uint32_t r[32];
            lcd::tmem_ld_32x32b_x32(lane_base + acc * BN + g * 32, r);
            lcd::tmem_ld_wait();
            emit(r, tn * BN + g * 32);
          }
        }
        lcd::tc_fence_before();
        // TWO_SM: the leader's MMAs refill both CTAs' accumulators, so both release on its
        // barrier.  One arrival per warp once every lane's TMEM reads are done (128 remote
        // arrivals per unit from the peer held the leader's next MMAs back by 2-4 us)
        __syncwarp();
        if (lane == 0) {
          if (!is_leader) lcd::mbar_arrive_remote(lcd::rank_addr(lcd::smem_u32(&tempty[acc]), leader));
          else lcd::mbar_arrive(&tempty[acc]);
        }
        h++;
      }
      if (split_mode && p.fixup) {
        // Split-K fixup without a second launch.  Each epilogue warp owns 32 rows of the tile:
        // it publishes its partial rows, counts its arrival on the (tile, warp) counter, and the
        // warp whose arrival completes the count sums all splits' partial rows in split order
        // (the same order whoever arrives last, so the result is deterministic) and stores C.
        // No warp ever waits for another.
        __threadfence();
        __syncwarp();
        const int32_t slot = ((b * p.tiles_m + tm) * p.tiles_n + tn) * 4 + q;
        uint32_t last = 0;
        if (lane == 0) last = atomicAdd(&p.counters[slot], 1) == p.splits - 1 ? 1u : 0u;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          if (m < p.M) {
#pragma unroll 1
            for (int g = 0; g < BN / 32; g++) {
              const int32_t n0 = tn * BN + g * 32;
              const int32_t cnt = min(32, p.N - n0);
              if (cnt <= 0) break;
              float v[32];
              sum_partials(p, v, b, m, n0, cnt);
              store_row<EPI>(p, v, c_row + (int64_t)n0 * p.c_ns, cnt);
            }
          }
          if (lane == 0) p.counters[slot] = 0;  // ready for the next launch that reuses the counters
        }
      }
    }
    // chain: this warp's part of product l is stored.  The four epilogue warps count themselves
    // in shared memory (they reach product l + 1 only after every CTA finished product l, so the
    // count goes up in whole groups of four) and the last of each group publishes the CTA to the
    // producers of product l + 1.
    if (src.counters() != nullptr) {
      __threadfence();
      __syncwarp();
      if (lane == 0 && (atomicAdd(layer_done, 1u) & 3u) == 3u)
        asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(src.counters() + l) : "memory");
    }
    }
  } else if constexpr (TF32X3) {
    // ---------------- 3xTF32 split ----------------
    // The tensor core reads a 32-bit operand as tf32 by ignoring its low 13 mantissa bits
    // (truncation: the f32 accuracy tests, 1e-5 normwise, would fail by an order of magnitude
    // if it rounded), so the raw f32 the TMA put in the stage serves unchanged as hi =
    // trunc(x).  lo = x - hi is exact in f32; it is rounded to tf32 here (nearest, ties away)
    // into the stage's lo half, so the tensor core reads it exactly.  Three products cannot
    // carry IEEE infinities (inf * hi(b) + inf * lo(b) is NaN when lo(b) = 0), so an infinite
    // or NaN x only marks the unit, whose epilogue then recomputes the tile exactly.
    const int ct = threadIdx.x - 192;  // 0 .. CONV_THREADS - 1
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    uint32_t uo = 0;  // unit ordinal
    for (int l = 0; ok && l < src.layers(); l++) {
    decltype(auto) p = src.kp(l);  // a chain's are copied to registers once per product
    for (int32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x, uo++) {
      int32_t b, split, tm, tn;
      unit_coords(p, u, &b, &split, &tm, &tn);
      const int32_t kb = split * p.kt_per_split;
      const int32_t ke = min(kb + p.kt_per_split, p.k_tiles);
      for (int32_t kt = kb; kt < ke; kt++) {
        if (!lcd::mbar_wait(&full[s], ph, p.err)) {
          ok = false;
          break;
        }
        // elementwise on identical layouts, so the swizzle is irrelevant
        const uint4* raw = reinterpret_cast<const uint4*>(a_hi(s));
        uint4* lo = reinterpret_cast<uint4*>(a_lo(s));
        constexpr int NV = (C::A_BYTES + C::B_BYTES) / 16;
        constexpr int CT = C::CONV_THREADS;
        static_assert(NV % (CT * 2) == 0, "converter passes of 2 vectors per thread");
#pragma unroll 1
        for (int v0 = ct; v0 < NV; v0 += CT * 2) {
          uint4 x[2];
#pragma unroll
          for (int q = 0; q < 2; q++) x[q] = raw[v0 + CT * q];
#pragma unroll
          for (int q = 0; q < 2; q++) {
            uint4 lv;
            const uint32_t* xs = reinterpret_cast<const uint32_t*>(&x[q]);
            uint32_t* ls = reinterpret_cast<uint32_t*>(&lv);
            uint32_t big = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float d = __fsub_rn(__uint_as_float(xs[e]), __uint_as_float(xs[e] & 0xffffe000u));
              ls[e] = (__float_as_uint(d) + 0x1000u) & 0xffffe000u;
              big = max(big, xs[e] & 0x7fffffffu);
            }
            if (big >= 0x7f800000u) {
              nonfinite[uo & 7] = uo + 1;
              __threadfence_block();
            }
            lo[v0 + CT * q] = lv;
          }
        }
        lcd::fence_proxy_async_smem();
        lcd::mbar_arrive(&conv[s]);
        if (++s == C::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    }
  }

  __syncthreads();
  // 2-SM: the peer's TMEM is written by the leader's MMAs; free it only once both CTAs are done
  if constexpr (TWO_SM) lcd::cluster_sync();
  if (warp == 1) {
    lcd::tc_fence_after();
    if constexpr (TWO_SM) lcd::tmem_dealloc_2sm(tmem_base, C::TMEM_COLS);
    else lcd::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  // neither CTA of a pair leaves while the other may still access its shared memory
  if constexpr (PAIR) lcd::cluster_sync();
}

template <int BN, bool TF32X3, int EPI, bool PAIR>
__global__ void __launch_bounds__(Cfg<BN, TF32X3, PAIR>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ KParams p) {
  gemm_body<BN, TF32X3, EPI, PAIR>(OneProduct{&tma_a, &tma_b, &p});
}

// 256 x 256 tiles over a cluster of 2 CTAs with cta_group::2 MMAs (16-bit inputs, no split).
template <int EPI>
__global__ void __launch_bounds__(Cfg<256, false, false, true>::THREADS, 1)
    gemm_2sm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    const __grid_constant__ KParams p) {
  gemm_body<256, false, EPI, false, OneProduct, true>(OneProduct{&tma_a, &tma_b, &p});
}

// 256 x 256 tiles over a cluster of 4: two CTA pairs with cta_group::2 MMAs, each summing one half
// of K, exchanging partials through distributed shared memory (16-bit inputs, 2-way split).
template <int EPI>
__global__ void __launch_bounds__(Cfg<256, false, true, true>::THREADS, 1)
    gemm_quad_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ KParams p) {
  gemm_body<256, false, EPI, true, OneProduct, true>(OneProduct{&tma_a, &tma_b, &p});
}

// A chain of skinny products (BN = 64, 16-bit inputs, CTA pairs): the pipeline's layer loop of
// one microbatch in one cooperative launch.
template <int EPI>
__global__ void __launch_bounds__(Cfg<64, false, true>::THREADS, 1)
    gemm_chain_kernel(const __grid_constant__ ChainParams cp) {
  gemm_body<64, false, EPI, true>(ChainSrc{&cp});
}

// ---- split-K reduce for many splits: C = epilogue(sum_s partial[s]) -------------------------------
// Used when so many splits share a tile that reducing inside the GEMM would serialise on a few
// warps.  kReduceChunks threads share each output quad (4 consecutive columns of one row,
// 16-byte partial loads): thread g sums the run of splits [g * c, (g + 1) * c), c =
// ceil(splits / kReduceChunks), in split order from +0 with its loads in flight ahead of the
// adds, and the quad's total is the run sums added in run order from +0.  Eight threads per
// quad keep a small output's partials in flight together; one thread walking all the splits
// waited out an L2 round trip per kReduceDepth splits.  The order depends only on the split
// count, so results are deterministic; up to kReduceChunks splits it is plain split order, the
// in-kernel fixup's.  Consecutive quads take consecutive rows when C's kernel rows are its
// contiguous axis (the swapped skinny products), consecutive column quads otherwise, so that
// C's stores coalesce either way.
constexpr int kReduceBlock = 128;
constexpr int kReduceChunks = 8;

template <int EPI>
__global__ void __launch_bounds__(kReduceBlock) splitk_reduce_kernel(const KParams p) {
  constexpr int kReduceDepth = 16;
  constexpr int kQuadsPerBlock = kReduceBlock / kReduceChunks;
  lcd::griddep_launch_dependents();
  lcd::griddep_wait();  // the partials are the GEMM's output
  const int32_t nq = (p.N + 3) / 4;  // column quads per row
  const int64_t rows = (int64_t)p.batch * p.M;
  const int64_t total = rows * nq;
  const int64_t plane = rows * (int64_t)p.N;
  const bool vec = (p.N % 4) == 0;
  const bool rows_fast = p.c_ms == 1 && p.c_ns != 1;
  const int g = threadIdx.x % kReduceChunks;
  const int32_t run = (p.splits + kReduceChunks - 1) / kReduceChunks;
  const int32_t s_begin = min(p.splits, g * run), s_end = min(p.splits, s_begin + run);
  // the loop bound is block-uniform, so every lane reaches the shuffles of every pass
  for (int64_t i0 = (int64_t)blockIdx.x * kQuadsPerBlock; i0 < total; i0 += (int64_t)gridDim.x * kQuadsPerBlock) {
    const int64_t i = i0 + threadIdx.x / kReduceChunks;
    const bool active = i < total;
    int64_t row = 0;
    int32_t quad = 0;
    if (!active) {
    } else if (rows_fast) {
      const int64_t bq = i / p.M;  // (batch, quad) pair
      const int32_t m = (int32_t)(i - bq * p.M);
      const int64_t b = bq / nq;
      quad = (int32_t)(bq - b * nq);
      row = b * p.M + m;
    } else {
      row = i / nq;
      quad = (int32_t)(i - row * nq);
    }
    const int32_t n0 = quad * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const float* src = p.partial + row * p.N + n0;
    if (active && vec) {
#pragma unroll 1
      for (int s0 = s_begin; s0 < s_end; s0 += kReduceDepth) {
        float4 v[kReduceDepth];
        const float* sp = src + (int64_t)s0 * plane;
#pragma unroll
        for (int u = 0; u < kReduceDepth; u++, sp += plane)
          if (s0 + u < s_end) v[u] = __ldcs(reinterpret_cast<const float4*>(sp));
#pragma unroll
        for (int u = 0; u < kReduceDepth; u++) {
          if (s0 + u < s_end) {
            acc[0] = __fadd_rn(acc[0], v[u].x);
            acc[1] = __fadd_rn(acc[1], v[u].y);
            acc[2] = __fadd_rn(acc[2], v[u].z);
            acc[3] = __fadd_rn(acc[3], v[u].w);
          }
        }
      }
    } else if (active) {
      for (int s = s_begin; s < s_end; s++)
        for (int e = 0; e < 4 && n0 + e < p.N; e++) acc[e] = __fadd_rn(acc[e], src[(int64_t)s * plane + e]);
    }
    // the runs' sums in run order from +0 (a run past the last split adds +0, which changes no
    // sum that started from +0)
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kReduceChunks; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) tot[e] = __fadd_rn(tot[e], __shfl_sync(0xffffffffu, acc[e], j, kReduceChunks));
    if (!active || g != 0) continue;
    const int32_t b = (int32_t)(row / p.M), m = (int32_t)(row - (int64_t)b * p.M);
    const int64_t base = p.c_off + (int64_t)b * p.c_bs + (int64_t)m * p.c_ms;
    float old[4];
#pragma unroll
    for (int e = 0; e < 4; e++)
      old[e] = n0 + e < p.N ? read_old<EPI>(p, base + (int64_t)(n0 + e) * p.c_ns) : 0.0f;
#pragma unroll
    for (int e = 0; e < 4; e++)
      if (n0 + e < p.N) write_new<EPI>(p, base + (int64_t)(n0 + e) * p.c_ns, tot[e], old[e]);
  }
}

// ---- C = beta * C (or zeros when beta == 0): the Fill plan ----------------------------------------
__global__ void __launch_bounds__(256) fill_kernel(KParams p) {
  const int64_t per = (int64_t)p.M * p.N;
  const int64_t total = per * p.batch;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t b = i / per;
    const int64_t rem = i - b * per;
    const int64_t m = rem / p.N, n = rem - m * p.N;
    const int64_t idx = p.c_off + b * p.c_bs + m * p.c_ms + n * p.c_ns;
    float v = 0.0f;
    if (p.beta != 0.0f) v = __fmul_rn(p.beta, load_c(p, idx));
    store_c(p, idx, v);
  }
}

// ---- host: tensor maps -----------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Encoded maps are cached by everything that goes into them (a map holds only the address,
// extents, strides, box and swizzle), so repeated products on the same buffers, such as a
// pipeline's GEMMs every step, skip the driver call.
struct MapKey {
  const void* base;
  uint64_t inner, rows, batch, rs, bs;
  uint32_t bi, br;
  int dt;
  bool atom32;
  bool operator==(const MapKey& o) const {
    return base == o.base && inner == o.inner && rows == o.rows && batch == o.batch && rs == o.rs && bs == o.bs &&
           bi == o.bi && br == o.br && dt == o.dt && atom32 == o.atom32;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = reinterpret_cast<uintptr_t>(k.base);
    for (uint64_t v : {k.inner, k.rows, k.batch, k.rs, k.bs, (uint64_t)k.bi << 32 | k.br,
                       (uint64_t)k.dt << 1 | (k.atom32 ? 1u : 0u)})
      h = (h ^ v) * 0x100000001b3ull;
    return (size_t)h;
  }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;
constexpr size_t kMapCacheMax = 16384;

// 3-D map over (packed axis, row axis, batch) with a 128-byte-swizzled box of box_inner x box_rows.
// `atom32` selects the 32-byte-atom variant of the 128-byte swizzle (MN-major f32 tiles).
lc_status make_map(CUtensorMap* map, const void* base, int in_dtype, uint64_t inner, uint64_t rows,
                   uint64_t batch, uint64_t row_stride_b, uint64_t batch_stride_b, uint32_t box_inner,
                   uint32_t box_rows, bool atom32 = false) {
  const MapKey key{base, inner, rows, batch, row_stride_b, batch_stride_b, box_inner, box_rows, in_dtype, atom32};
  {
    std::lock_guard<std::mutex> g(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *map = it->second;
      return LC_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return lc::fail(LC_ERR_LAUNCH, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMapDataType dt = in_dtype == LC_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : in_dtype == LC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {inner, rows, batch};
  cuuint64_t strides[2] = {row_stride_b, batch_stride_b};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return lc::fail(LC_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  std::lock_guard<std::mutex> g(g_map_mu);
  if (g_maps.size() >= kMapCacheMax) g_maps.clear();
  g_maps.emplace(key, *map);
  return LC_OK;
}

template <int BN, bool TF32X3, int EPI, bool PAIR>
cudaLaunchConfig_t launch_config(cudaStream_t s, int grid, cudaLaunchAttribute (&at)[2]) {
  using C = Cfg<BN, TF32X3, PAIR>;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  int na = 0;
  // programmatic dependent launch: this grid's set-up may overlap the previous kernel's tail
  at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[na].val.programmaticStreamSerializationAllowed = 1;
  na++;
  if (PAIR) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = 2;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  return cfg;
}

template <int BN, bool TF32X3, int EPI, bool PAIR>
lc_status prepare_kernel(lc_context* ctx) {
  using C = Cfg<BN, TF32X3, PAIR>;
  static bool attr_set[64] = {false};
  if (!attr_set[ctx->device % 64]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, TF32X3, EPI, PAIR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return lc::cuda_fail(e, "cudaFuncSetAttribute(gemm)");
    attr_set[ctx->device % 64] = true;
  }
  return LC_OK;
}

// How many CTA pairs of this kernel fit on the device at once (0 when pairs cannot launch).
template <int BN, int EPI>
int pair_capacity(lc_context* ctx) {
  static int cap[64];
  static bool known[64] = {false};
  const int d = ctx->device % 64;
  if (!known[d]) {
    int n = 0;
    if (prepare_kernel<BN, false, EPI, true>(ctx) == LC_OK) {
      cudaLaunchAttribute at[2];
      cudaLaunchConfig_t cfg = launch_config<BN, false, EPI, true>(nullptr, 2, at);
      if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<BN, false, EPI, true>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    cap[d] = n;
    known[d] = true;
  }
  return cap[d];
}

template <int BN, bool TF32X3, int EPI, bool PAIR>
lc_status launch_kernel(lc_context* ctx, cudaStream_t s, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& p,
                        int grid) {
  lc_status st = prepare_kernel<BN, TF32X3, EPI, PAIR>(ctx);
  if (st) return st;
  cudaLaunchAttribute at[2];
  cudaLaunchConfig_t cfg = launch_config<BN, TF32X3, EPI, PAIR>(s, grid, at);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, TF32X3, EPI, PAIR>, ta, tb, p);
  lc::record_launch(ctx, PAIR ? (BN == 64 ? "gemm_bf16_pair_n64" : BN == 128 ? "gemm_bf16_pair_n128" : "gemm_bf16_pair_n256")
                         : TF32X3 ? (BN == 64 ? "gemm_tf32x3_n64" : "gemm_tf32x3_n128")
                                  : (BN == 64 ? "gemm_bf16_n64" : BN == 128 ? "gemm_bf16_n128" : "gemm_bf16_n256"));
  if (e != cudaSuccess) return lc::cuda_fail(e, "gemm launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return lc::cuda_fail(e, "gemm launch");
  return LC_OK;
}

template <int EPI>
cudaLaunchConfig_t launch_config_2sm(cudaStream_t s, int grid, cudaLaunchAttribute (&at)[2]) {
  using C = Cfg<256, false, false, true>;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = 2;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cfg;
}

template <int EPI>
lc_status prepare_2sm(lc_context* ctx) {
  static bool attr_set[64] = {false};
  if (!attr_set[ctx->device % 64]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_2sm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg<256, false, false, true>::SMEM);
    if (e != cudaSuccess) return lc::cuda_fail(e, "cudaFuncSetAttribute(gemm 2sm)");
    attr_set[ctx->device % 64] = true;
  }
  return LC_OK;
}

// How many 2-SM clusters fit on the device at once (0 when they cannot launch).
template <int EPI>
int capacity_2sm(lc_context* ctx) {
  static int cap[64];
  static bool known[64] = {false};
  const int d = ctx->device % 64;
  if (!known[d]) {
    int n = 0;
    if (prepare_2sm<EPI>(ctx) == LC_OK) {
      cudaLaunchAttribute at[2];
      cudaLaunchConfig_t cfg = launch_config_2sm<EPI>(nullptr, 2, at);
      if (cudaOccupancyMaxActiveClusters(&n, gemm_2sm_kernel<EPI>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    cap[d] = n;
    known[d] = true;
  }
  return cap[d];
}

template <int EPI>
lc_status launch_2sm(lc_context* ctx, cudaStream_t s, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& p,
                     int grid) {
  lc_status st = prepare_2sm<EPI>(ctx);
  if (st) return st;
  cudaLaunchAttribute at[2];
  cudaLaunchConfig_t cfg = launch_config_2sm<EPI>(s, grid, at);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_2sm_kernel<EPI>, ta, tb, p);
  lc::record_launch(ctx, "gemm_bf16_2sm_n256");
  if (e != cudaSuccess) return lc::cuda_fail(e, "gemm 2sm launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return lc::cuda_fail(e, "gemm 2sm launch");
  return LC_OK;
}

template <int EPI>
cudaLaunchConfig_t launch_config_quad(cudaStream_t s, int grid, cudaLaunchAttribute (&at)[2]) {
  cudaLaunchConfig_t cfg = launch_config_2sm<EPI>(s, grid, at);
  cfg.dynamicSmemBytes = Cfg<256, false, true, true>::SMEM;
  at[1].val.clusterDim.x = 4;
  return cfg;
}

template <int EPI>
lc_status prepare_quad(lc_context* ctx) {
  static bool attr_set[64] = {false};
  if (!attr_set[ctx->device % 64]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_quad_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg<256, false, true, true>::SMEM);
    if (e != cudaSuccess) return lc::cuda_fail(e, "cudaFuncSetAttribute(gemm quad)");
    attr_set[ctx->device % 64] = true;
  }
  return LC_OK;
}

// How many clusters of 4 fit on the device at once (0 when they cannot launch).
template <int EPI>
int capacity_quad(lc_context* ctx) {
  static int cap[64];
  static bool known[64] = {false};
  const int d = ctx->device % 64;
  if (!known[d]) {
    int n = 0;
    if (prepare_quad<EPI>(ctx) == LC_OK) {
      cudaLaunchAttribute at[2];
      cudaLaunchConfig_t cfg = launch_config_quad<EPI>(nullptr, 4, at);
      if (cudaOccupancyMaxActiveClusters(&n, gemm_quad_kernel<EPI>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    cap[d] = n;
    known[d] = true;
  }
  return cap[d];
}

template <int EPI>
lc_status launch_quad(lc_context* ctx, cudaStream_t s, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& p,
                      int grid) {
  lc_status st = prepare_quad<EPI>(ctx);
  if (st) return st;
  cudaLaunchAttribute at[2];
  cudaLaunchConfig_t cfg = launch_config_quad<EPI>(s, grid, at);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_quad_kernel<EPI>, ta, tb, p);
  lc::record_launch(ctx, "gemm_bf16_quad_n256");
  if (e != cudaSuccess) return lc::cuda_fail(e, "gemm quad launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return lc::cuda_fail(e, "gemm quad launch");
  return LC_OK;
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace

namespace lc {

bool tma_operand_ok(const GemmOperand& o, int in_dtype) {
  const size_t es = dtype_size(in_dtype);
  const uintptr_t base = reinterpret_cast<uintptr_t>(o.data) + o.offset * es;
  if (base % 16) return false;
  const int major = operand_major(o);
  if (major < 0) return false;
  // the row axis (the one that is not packed) and the batch axis need 16-byte multiple,
  // non-zero strides unless their extent is 1
  const int64_t row_stride = major == 0 ? o.mn_stride : o.k_stride;
  const uint64_t rows = major == 0 ? o.mn : o.k;
  if (rows > 1 && (row_stride <= 0 || ((uint64_t)row_stride * es) % 16 != 0)) return false;
  if (o.batch > 1 && (o.batch_stride <= 0 || ((uint64_t)o.batch_stride * es) % 16 != 0)) return false;
  if (o.mn >= (1ull << 31) || o.k >= (1ull << 31) || o.batch >= (1ull << 31)) return false;
  return true;
}

}  // namespace lc

namespace {

// Everything a launch of one product needs, decided once: orientation, tile width, split,
// CTA pairs, tensor maps and the kernel parameters.
struct Planned {
  KParams p{};
  CUtensorMap ta, tb;
  int bn = 64;
  bool tf32x3 = false, pair = false, two_sm = false, quad = false;
  int64_t pair_clusters = 0, two_sm_clusters = 0, quad_clusters = 0, tiles = 0, units = 0, splits = 1, M = 0, N = 0;
  bool swap = false;
};

lc_status plan_gemm(lc_context* ctx, const lc::GemmProblem& pr, lc_contract_plan* plan, bool dry_run, Planned* out) {
  using namespace lc;
  GemmOperand A = pr.a, B = pr.b;
  uint64_t M = pr.m, N = pr.n;
  int64_t c_ms = pr.c_m_stride, c_ns = pr.c_n_stride;
  bool swap = false;
  // Skinny M: compute C^T = B^T A^T so the long side fills the 128-row MMA.
  if (pr.swap_hint != 0 ? pr.swap_hint > 0 : (M < 128 && N > M)) {
    std::swap(A, B);
    std::swap(M, N);
    std::swap(c_ms, c_ns);
    swap = true;
  }
  const bool tf32x3 = pr.in_dtype == LC_F32;
  const int epr = tf32x3 ? 32 : 64;
  const size_t es = dtype_size(pr.in_dtype);
  int bn = N <= 64 ? 64 : (N <= 128 || tf32x3) ? 128 : 256;
  if (!tf32x3 && (pr.bn_hint == 64 || pr.bn_hint == 128 || pr.bn_hint == 256)) bn = pr.bn_hint;
  const int64_t tiles_m = ceil_div(M, 128);
  const int64_t k_tiles = ceil_div(pr.k, epr);
  // Split-K choice: the CTAs are persistent, one per SM, so a unit count just above a multiple
  // of the SM count costs a whole extra wave.  Cost of s splits, in k-tile times along the
  // critical path: waves(s) * (k-tiles per unit + the unit's partial write and reduce read,
  // expressed in k-tile loads).  The cheapest s wins; ties go to fewer splits.
  const int64_t sms = std::max<int64_t>(1, ctx->sm_count - pr.reserve_sms);
  static const int64_t env_splits = [] {
    const char* e = getenv("LC_SPLITK");  // tuning override for sweeps; unset in normal use
    return e ? atoll(e) : 0ll;
  }();
  auto best_split = [&](int bn_try, int64_t* s_out) -> double {
    const int64_t t = tiles_m * ceil_div(N, bn_try) * pr.batch;
    const double partial_cost = (128.0 * bn_try * 4.0 * 2.0) / ((double)(128 + bn_try) * 128.0);
    auto split_cost = [&](int64_t sp) {
      const int64_t per = ceil_div(k_tiles, sp);
      const int64_t real = ceil_div(k_tiles, per);
      const int64_t waves = ceil_div(t * real, sms);
      return (double)waves * ((double)per + (real > 1 ? partial_cost : 0.0));
    };
    int64_t sp = 1;
    double best = split_cost(1);
    if (pr.splits_hint > 0 || env_splits > 0) {
      sp = std::max<int64_t>(1, std::min<int64_t>(pr.splits_hint > 0 ? pr.splits_hint : env_splits, k_tiles));
      best = split_cost(sp);
    } else {
      for (int64_t c = 2; c <= std::min<int64_t>(k_tiles, 512); c++) {
        const double v = split_cost(c);
        if (v < best * 0.999) {
          best = v;
          sp = c;
        }
      }
    }
    *s_out = sp;
    return best;
  };
  int64_t splits = 1, kps = k_tiles;
  const double cost = best_split(bn, &splits);
  // 3xTF32: a 128 x 64 tile's k-tile takes about 0.6 of a 128 x 128 one (the converters' and the
  // MMAs' work on B halves, on A it does not), so the narrower tile wins when it spares a split
  // or a wave: the 1024^3 product runs unsplit on 128 x 64 tiles in 31.8 us, against 36.1 us
  // with two splits on 128 x 128 (same-box timings)
  if (tf32x3 && bn == 128 && pr.bn_hint == 0) {
    int64_t s64 = 1;
    const double c64 = 0.6 * best_split(64, &s64);
    if (c64 < cost * 0.999) {
      bn = 64;
      splits = s64;
    }
  }
  const int64_t tiles_n = ceil_div(N, bn);
  const int64_t tiles = tiles_m * tiles_n * pr.batch;
  splits = std::max<int64_t>(splits, 1);
  kps = ceil_div(k_tiles, splits);
  splits = ceil_div(k_tiles, kps);
  const int64_t units = tiles * splits;
  // A 2-way split of 16-bit inputs runs as CTA pairs (clusters of 2) that reduce through
  // distributed shared memory: no partial sums in global memory, no second pass.
  static const bool env_no_pair = [] {
    const char* e = getenv("LC_GEMM_PAIRS");  // tuning override: "0" keeps 2-way splits in global memory
    return e != nullptr && e[0] == '0';
  }();
  int64_t pair_clusters = 0;
  if (!dry_run && !tf32x3 && splits == 2 && pr.epi != 2 && !env_no_pair) {
    const int cap = bn == 64    ? (pr.epi == 0 ? pair_capacity<64, 0>(ctx) : pair_capacity<64, 1>(ctx))
                    : bn == 128 ? (pr.epi == 0 ? pair_capacity<128, 0>(ctx) : pair_capacity<128, 1>(ctx))
                                : (pr.epi == 0 ? pair_capacity<256, 0>(ctx) : pair_capacity<256, 1>(ctx));
    pair_clusters = std::min<int64_t>({tiles, (int64_t)cap, (ctx->sm_count - pr.reserve_sms) / 2});
  }
  const bool pair = pair_clusters > 0;
  // A 2-way split of a 256-wide tile with at least 256 rows runs on clusters of 4: two CTA pairs
  // with cta_group::2 MMAs over 256 x 256 tiles, one pair per K half, exchanging partials like a
  // CTA pair.  Each CTA loads 128 rows of A and half of B^T per stage, a third less than a
  // 128 x 256 tile on one SM, which is what bounds the grouped skinny products.
  static const bool env_no_quad = [] {
    const char* e = getenv("LC_GEMM_QUAD");  // tuning override: "0" keeps such products on CTA pairs
    return e != nullptr && e[0] == '0';
  }();
  int64_t quad_clusters = 0;
  if (pair && bn == 256 && M >= 256 && !env_no_quad) {
    const int cap = pr.epi == 0 ? capacity_quad<0>(ctx) : capacity_quad<1>(ctx);
    quad_clusters = std::min<int64_t>({ceil_div(M, 256) * ceil_div(N, bn) * (int64_t)pr.batch, (int64_t)cap,
                                       (ctx->sm_count - pr.reserve_sms) / 4});
  }
  const bool quad = quad_clusters > 0;
  // 256-row tiles over CTA pairs (cta_group::2 MMAs): each CTA reads 128 rows of A and half of
  // the tile's B^T, a third less operand traffic per output than a 128 x 256 tile on one SM.
  // Taken for unsplit BN = 256 products with enough tiles to give every pair of SMs work.
  static const bool env_no_2sm = [] {
    const char* e = getenv("LC_GEMM_2SM");  // tuning override: "0" keeps 128-row tiles on one SM
    return e != nullptr && e[0] == '0';
  }();
  const int64_t tiles_m2 = ceil_div(M, 256);
  const int64_t tiles2 = tiles_m2 * tiles_n * pr.batch;
  const int64_t sm_pairs = (ctx->sm_count - pr.reserve_sms) / 2;
  int64_t two_sm_clusters = 0;
  if (!dry_run && !tf32x3 && !pair && splits == 1 && bn == 256 && M >= 256 && tiles2 >= sm_pairs && !env_no_2sm) {
    const int cap = pr.epi == 0 ? capacity_2sm<0>(ctx) : pr.epi == 1 ? capacity_2sm<1>(ctx) : capacity_2sm<2>(ctx);
    two_sm_clusters = std::min<int64_t>({tiles2, (int64_t)cap, sm_pairs});
  }
  const bool two_sm = two_sm_clusters > 0;
  const int64_t tiles_m_eff = (two_sm || quad) ? tiles_m2 : tiles_m;
  const int64_t units_eff = two_sm ? tiles2 : quad ? tiles2 * splits : units;
  if (units >= (1ll << 31) || k_tiles >= (1ll << 31)) return fail(LC_ERR_INVALID_ARGUMENT, "problem too large");

  if (operand_major(A) < 0 || operand_major(B) < 0) return fail(LC_ERR_INVALID_ARGUMENT, "operand has no unit stride");
  const bool a_mn = operand_major(A) == 1;
  const bool b_mn = operand_major(B) == 1;
  if (plan) {
    plan->kind = splits > 1 ? 3 : 2;
    plan->splits = (int32_t)splits;
    plan->batch = pr.batch;
    plan->m = pr.m;
    plan->n = pr.n;
    plan->k = pr.k;
    plan->swap_ab = swap ? 1 : 0;
    plan->a_major = a_mn ? 1 : 0;
    plan->b_major = b_mn ? 1 : 0;
  }
  if (dry_run) return LC_OK;

  CUtensorMap& ta = out->ta;
  CUtensorMap& tb = out->tb;
  lc_status st;
  const void* abase = static_cast<const uint8_t*>(A.data) + A.offset * es;
  const void* bbase = static_cast<const uint8_t*>(B.data) + B.offset * es;
  auto bstride = [&](const GemmOperand& o, uint64_t fallback) -> uint64_t {
    return o.batch > 1 ? o.batch_stride * es : fallback;
  };
  if (!a_mn) {
    uint64_t rs = A.mn > 1 ? A.mn_stride * es : ((A.k * es + 15) / 16) * 16;
    st = make_map(&ta, abase, pr.in_dtype, A.k, A.mn, pr.batch, rs, bstride(A, rs * A.mn), epr, 128);
  } else {
    uint64_t rs = A.k > 1 ? A.k_stride * es : ((A.mn * es + 15) / 16) * 16;
    st = make_map(&ta, abase, pr.in_dtype, A.mn, A.k, pr.batch, rs, bstride(A, rs * A.k), epr, epr, tf32x3);
  }
  if (st) return st;
  if (!b_mn) {
    uint64_t rs = B.mn > 1 ? B.mn_stride * es : ((B.k * es + 15) / 16) * 16;
    st = make_map(&tb, bbase, pr.in_dtype, B.k, B.mn, pr.batch, rs, bstride(B, rs * B.mn), epr,
                  (two_sm || quad) ? bn / 2 : bn);
  } else {
    uint64_t rs = B.k > 1 ? B.k_stride * es : ((B.mn * es + 15) / 16) * 16;
    st = make_map(&tb, bbase, pr.in_dtype, B.mn, B.k, pr.batch, rs, bstride(B, rs * B.k), epr, epr, tf32x3);
  }
  if (st) return st;

  KParams& p = out->p;
  p = KParams{};
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.k_tiles = (int32_t)k_tiles;
  p.kt_per_split = (int32_t)kps;
  p.splits = (int32_t)splits;
  p.batch = (int32_t)pr.batch;
  p.tiles_m = (int32_t)tiles_m_eff;
  p.tiles_n = (int32_t)tiles_n;
  p.units = (int32_t)units_eff;
  p.split_minor = pair ? 1 : 0;
  static const bool env_no_hint = [] {
    const char* e = getenv("LC_GEMM_EVICT_FIRST");  // tuning override: "0" drops the streaming hint
    return e != nullptr && e[0] == '0';
  }();
  p.a_once = (tiles_n == 1 && !env_no_hint) ? 1 : 0;
  p.b_once = (tiles_m_eff == 1 && !env_no_hint) ? 1 : 0;
  static const int env_prefetch = [] {
    const char* e = getenv("LC_GEMM_PREFETCH");  // tuning override: k-tiles of L2 prefetch ahead (0 = off)
    return e ? atoi(e) : -1;
  }();
  // L2 prefetch of the streamed operand (16-bit CTA-pair products, whose A is the weight matrix
  // of the pipeline's skinny and grouped products)
  p.prefetch = (pair && !tf32x3) ? (env_prefetch >= 0 ? env_prefetch : kPrefetchTiles) : 0;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  const uint32_t fmt = tf32x3 ? 2u : (pr.in_dtype == LC_BF16 ? 1u : 0u);
  p.idesc = lcd::make_idesc(fmt, (two_sm || quad) ? 256 : 128, bn, a_mn, b_mn);
  p.c_dtype = pr.c_dtype;
  p.relu = pr.relu;
  p.c = pr.c;
  p.c_off = (int64_t)pr.c_offset;
  p.c_bs = pr.c_batch_stride;
  p.c_ms = c_ms;
  p.c_ns = c_ns;
  p.alpha = pr.alpha;
  p.beta = pr.beta;
  p.err = ctx->d_error;
  if (tf32x3) {
    p.fa = static_cast<const float*>(A.data) + A.offset;
    p.fb = static_cast<const float*>(B.data) + B.offset;
    p.fa_ms = A.mn_stride;
    p.fa_ks = A.k_stride;
    p.fa_bs = A.batch > 1 ? A.batch_stride : 0;
    p.fb_ns = B.mn_stride;
    p.fb_ks = B.k_stride;
    p.fb_bs = B.batch > 1 ? B.batch_stride : 0;
    p.K = (int64_t)pr.k;
  }
  if (tf32x3 && (pr.epi == 1 || pr.epi == 2))
    return fail(LC_ERR_INVALID_ARGUMENT, "the mask and SGD epilogues take 16-bit inputs");
  if (!tf32x3 && pr.epi >= 3) return fail(LC_ERR_INVALID_ARGUMENT, "the GELU epilogues take f32 inputs");
  if (pr.epi < 0 || pr.epi > 4) return fail(LC_ERR_INVALID_ARGUMENT, "unknown epilogue");
  {
    // 16-byte vector epilogue: C's columns contiguous, every row start a multiple of 8 elements
    // from 16-byte-aligned bases (8 covers both 2- and 4-byte elements)
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool strides8 = (p.c_off % 8) == 0 && (p.c_ms % 8) == 0 && (pr.batch == 1 || (p.c_bs % 8) == 0);
    const bool ptrs = pr.epi == 0   ? al16(pr.c)
                      : pr.epi == 1 ? al16(pr.c) && al16(pr.aux)
                      : pr.epi == 2 ? al16(pr.aux) && al16(pr.aux2)
                      : pr.epi == 3 ? al16(pr.c) && (pr.aux2 == nullptr || al16(pr.aux2))
                                    : al16(pr.c) && al16(pr.aux);
    p.vec = (c_ns == 1 && strides8 && ptrs) ? 1 : 0;
    const bool tstrides8 = (p.c_off % 8) == 0 && (p.c_ns % 8) == 0 && (pr.batch == 1 || (p.c_bs % 8) == 0);
    p.tvec = (c_ms == 1 && c_ns != 1 && tstrides8 && ptrs && pr.epi != 2) ? 1 : 0;
  }
  p.aux = pr.aux;
  p.aux2 = pr.aux2;
  p.lr = pr.lr;
  out->bn = bn;
  out->tf32x3 = tf32x3;
  out->pair = pair;
  out->pair_clusters = pair_clusters;
  out->two_sm = two_sm;
  out->two_sm_clusters = two_sm_clusters;
  out->quad = quad;
  out->quad_clusters = quad_clusters;
  out->tiles = (two_sm || quad) ? tiles2 : tiles;
  out->units = units_eff;
  out->splits = splits;
  out->M = (int64_t)M;
  out->N = (int64_t)N;
  out->swap = swap;
  return LC_OK;
}

}  // namespace

namespace lc {

lc_status gemm_run(lc_context* ctx, cudaStream_t s, const GemmProblem& pr, lc_contract_plan* plan, bool dry_run) {
  Planned pl;
  lc_status st = plan_gemm(ctx, pr, plan, dry_run, &pl);
  if (st || dry_run) return st;
  KParams& p = pl.p;
  const CUtensorMap& ta = pl.ta;
  const CUtensorMap& tb = pl.tb;
  const int bn = pl.bn;
  const bool tf32x3 = pl.tf32x3, pair = pl.pair;
  const int64_t pair_clusters = pl.pair_clusters, tiles = pl.tiles, units = pl.units, splits = pl.splits;
  const uint64_t M = (uint64_t)pl.M, N = (uint64_t)pl.N;
  // Split-K scratch: the partial tiles and, for the in-kernel fixup (up to kFixupMaxSplits splits,
  // where each reducing warp sums few partials), one arrival counter per (batch, tile, epilogue
  // warp).  On the context's own stream the context keeps both between calls (its counters are
  // zero between launches: each fixup resets what it used); on any other stream they come from
  // the stream-ordered pool, counters zeroed in stream order.
  constexpr int64_t kFixupMaxSplits = 4;
  void* scratch = nullptr;
  if (splits > 1 && !pair) {
    p.fixup = splits <= kFixupMaxSplits ? 1 : 0;
    const size_t part_bytes = sizeof(float) * (size_t)splits * pr.batch * M * N;
    const size_t part_pad = (part_bytes + 255) / 256 * 256;
    const size_t cnt_n = (size_t)tiles * 4;
    if (pr.fixed_part != nullptr) {
      if (part_bytes > pr.fixed_part_bytes)
        return fail(LC_ERR_INVALID_ARGUMENT, "split-K partials need " + std::to_string(part_bytes) +
                                                 " bytes; the fixed scratch holds " +
                                                 std::to_string(pr.fixed_part_bytes));
      if (p.fixup && cnt_n > pr.fixed_cnt_n)
        return fail(LC_ERR_INVALID_ARGUMENT, "split-K fixup needs " + std::to_string(cnt_n) +
                                                 " tile counters; the fixed scratch holds " +
                                                 std::to_string(pr.fixed_cnt_n));
      p.partial = pr.fixed_part;
      p.counters = pr.fixed_cnt;
      // the fixup's arrival counters must start at zero
      if (p.fixup) {
        cudaError_t e = cudaMemsetAsync(p.counters, 0, cnt_n * sizeof(int), s);
        if (e != cudaSuccess) return cuda_fail(e, "split-K counters");
      }
    } else if (s == ctx->stream) {
      if (ctx->split_part_bytes < part_pad || ctx->split_cnt_n < cnt_n) {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e == cudaSuccess && ctx->split_part_bytes < part_pad) {
          if (ctx->split_part) cudaFree(ctx->split_part);
          ctx->split_part = nullptr;
          ctx->split_part_bytes = 0;
          e = cudaMalloc(&ctx->split_part, part_pad);
          if (e == cudaSuccess) ctx->split_part_bytes = part_pad;
        }
        if (e == cudaSuccess && ctx->split_cnt_n < cnt_n) {
          if (ctx->split_cnt) cudaFree(ctx->split_cnt);
          ctx->split_cnt = nullptr;
          ctx->split_cnt_n = 0;
          const size_t n = std::max<size_t>(cnt_n, 4096);
          e = cudaMalloc(&ctx->split_cnt, n * sizeof(int));
          if (e == cudaSuccess) e = cudaMemsetAsync(ctx->split_cnt, 0, n * sizeof(int), s);
          if (e == cudaSuccess) ctx->split_cnt_n = n;
        }
        if (e != cudaSuccess) return cuda_fail(e, "split-K scratch");
      }
      p.partial = static_cast<float*>(ctx->split_part);
      p.counters = ctx->split_cnt;
    } else {
      st = scratch_alloc(ctx, s, part_pad + cnt_n * sizeof(int), &scratch);
      if (st) return st;
      p.partial = static_cast<float*>(scratch);
      p.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + part_pad);
      cudaError_t e = p.fixup ? cudaMemsetAsync(p.counters, 0, cnt_n * sizeof(int), s) : cudaSuccess;
      if (e != cudaSuccess) {
        scratch_free(scratch, s);
        return cuda_fail(e, "split-K counters");
      }
    }
  }
  const int grid = pl.quad ? (int)(4 * pl.quad_clusters)
                   : pair ? (int)(2 * pair_clusters)
                   : pl.two_sm ? (int)(2 * pl.two_sm_clusters)
                               : (int)std::max<int64_t>(1, std::min<int64_t>(units, ctx->sm_count - pr.reserve_sms));
  if (pl.quad) {
    st = pr.epi == 0 ? launch_quad<0>(ctx, s, ta, tb, p, grid) : launch_quad<1>(ctx, s, ta, tb, p, grid);
  } else if (pl.two_sm) {
    st = pr.epi == 0   ? launch_2sm<0>(ctx, s, ta, tb, p, grid)
         : pr.epi == 1 ? launch_2sm<1>(ctx, s, ta, tb, p, grid)
                       : launch_2sm<2>(ctx, s, ta, tb, p, grid);
  } else if (pair) {
    st = bn == 64    ? (pr.epi == 0 ? launch_kernel<64, false, 0, true>(ctx, s, ta, tb, p, grid)
                                    : launch_kernel<64, false, 1, true>(ctx, s, ta, tb, p, grid))
         : bn == 128 ? (pr.epi == 0 ? launch_kernel<128, false, 0, true>(ctx, s, ta, tb, p, grid)
                                    : launch_kernel<128, false, 1, true>(ctx, s, ta, tb, p, grid))
                     : (pr.epi == 0 ? launch_kernel<256, false, 0, true>(ctx, s, ta, tb, p, grid)
                                    : launch_kernel<256, false, 1, true>(ctx, s, ta, tb, p, grid));
  } else if (tf32x3) {
    auto tf32_by_bn = [&](auto epi_tag) {
      constexpr int E = decltype(epi_tag)::value;
      return bn == 64 ? launch_kernel<64, true, E, false>(ctx, s, ta, tb, p, grid)
                      : launch_kernel<128, true, E, false>(ctx, s, ta, tb, p, grid);
    };
    st = pr.epi == 0   ? tf32_by_bn(std::integral_constant<int, 0>{})
         : pr.epi == 3 ? tf32_by_bn(std::integral_constant<int, 3>{})
                       : tf32_by_bn(std::integral_constant<int, 4>{});
  } else {
    auto by_bn = [&](auto epi_tag) {
      constexpr int E = decltype(epi_tag)::value;
      return bn == 64    ? launch_kernel<64, false, E, false>(ctx, s, ta, tb, p, grid)
             : bn == 128 ? launch_kernel<128, false, E, false>(ctx, s, ta, tb, p, grid)
                         : launch_kernel<256, false, E, false>(ctx, s, ta, tb, p, grid);
    };
    st = pr.epi == 0   ? by_bn(std::integral_constant<int, 0>{})
         : pr.epi == 1 ? by_bn(std::integral_constant<int, 1>{})
                       : by_bn(std::integral_constant<int, 2>{});
  }
  if (st == LC_OK && splits > 1 && !pair && !p.fixup) {
    const int64_t quads = (int64_t)pr.batch * M * ((N + 3) / 4);
    const int rgrid = (int)std::max<int64_t>(
        1, std::min<int64_t>(ceil_div(quads, kReduceBlock / kReduceChunks), (int64_t)ctx->sm_count * 16));
    // a programmatic dependent of the GEMM: its blocks are resident and waiting when the last
    // partial lands (measured 62.1 -> 60.3 us on the 256 x 256 x 262144 bf16 product)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)rgrid);
    cfg.blockDim = dim3(kReduceBlock);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = pr.epi == 0   ? cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<0>, p)
                    : pr.epi == 1 ? cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<1>, p)
                    : pr.epi == 2 ? cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<2>, p)
                    : pr.epi == 3 ? cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<3>, p)
                                  : cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<4>, p);
    record_launch(ctx, "gemm_splitk_reduce");
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) st = cuda_fail(e, "split-K reduce launch");
  }
  if (scratch) scratch_free(scratch, s);
  return st;
}

lc_status gemm_plan_shape(lc_context* ctx, const GemmProblem& pr, int32_t* bn, int32_t* splits, int32_t* swap) {
  Planned pl;
  lc_status st = plan_gemm(ctx, pr, nullptr, false, &pl);
  if (st) return st;
  *bn = pl.bn;
  *splits = (int32_t)pl.splits;
  *swap = pl.swap ? 1 : -1;
  return LC_OK;
}

lc_status gemm_chain_run(lc_context* ctx, cudaStream_t s, const GemmProblem* probs, int n, bool a_stable,
                         int max_clusters, bool* chained) {
  *chained = false;
  static const bool env_off = [] {
    const char* e = getenv("LC_GEMM_CHAIN");  // "0": run chains as separate launches
    return e != nullptr && e[0] == '0';
  }();
  if (env_off || n <= 0 || n > kMaxChain) return LC_OK;
  const int epi = probs[0].epi;
  if (epi != 0 && epi != 1) return LC_OK;
  thread_local std::unique_ptr<ChainParams> cp_holder;
  if (!cp_holder) cp_holder.reset(new ChainParams());
  ChainParams& cp = *cp_holder;
  int64_t clusters = 0, tiles = 0;
  for (int i = 0; i < n; i++) {
    if (probs[i].epi != epi) return LC_OK;
    Planned pl;
    lc_status st = plan_gemm(ctx, probs[i], nullptr, false, &pl);
    if (st) return st;
    if (!pl.pair || pl.bn != 64) return LC_OK;
    cp.p[i] = pl.p;
    cp.a[i] = pl.ta;
    cp.b[i] = pl.tb;
    clusters = std::max<int64_t>(clusters, pl.pair_clusters);
    tiles = std::max<int64_t>(tiles, pl.tiles);
  }
  if (max_clusters > 0 && clusters > max_clusters) {
    // as few waves as the cap allows, spread evenly over the pairs (counted in tiles, which can
    // outnumber the pairs that fit at once)
    const int64_t work = std::max<int64_t>(clusters, tiles);
    const int64_t waves = ceil_div(work, max_clusters);
    clusters = std::min<int64_t>(clusters, ceil_div(work, waves));
  }
  cp.n = n;
  cp.a_stable = a_stable ? 1 : 0;
  // counters per stream slot: chains on different streams may run at the same time
  int slot = -1;
  for (int i = 0; i < kChainStreams; i++)
    if (ctx->chain_stream[i] == s || ctx->chain_stream[i] == nullptr) {
      slot = i;
      break;
    }
  if (slot < 0) return LC_OK;  // more concurrent chain streams than slots: run the products one by one
  if (ctx->chain_cnt == nullptr) {
    cudaError_t e = cudaMalloc(&ctx->chain_cnt, kChainStreams * kMaxChain * sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "chain counters");
  }
  ctx->chain_stream[slot] = s;
  int* counters = ctx->chain_cnt + slot * kMaxChain;
  cp.counters = counters;
  cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)n * sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail(e, "chain counters");
  auto kern = epi == 0 ? gemm_chain_kernel<0> : gemm_chain_kernel<1>;
  using C = Cfg<64, false, true>;
  static bool attr_set[2][64] = {};
  if (!attr_set[epi][ctx->device % 64]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm chain)");
    attr_set[epi][ctx->device % 64] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * clusters));
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  // every CTA of the chain waits on every other between products: all must be resident at once
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = 2;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, cp);
  if (e != cudaSuccess) {
    // e.g. more clusters than can be co-resident: leave the chain to one-by-one launches
    cudaGetLastError();
    return LC_OK;
  }
  record_launch(ctx, epi == 0 ? "gemm_bf16_chain_n64" : "gemm_bf16_chain_mask_n64");
  *chained = true;
  return LC_OK;
}

lc_status gemm_fill(lc_context* ctx, cudaStream_t s, const GemmProblem& pr) {
  KParams p{};
  p.M = (int32_t)pr.m;
  p.N = (int32_t)pr.n;
  p.batch = (int32_t)pr.batch;
  p.c = pr.c;
  p.c_dtype = pr.c_dtype;
  p.c_off = (int64_t)pr.c_offset;
  p.c_bs = pr.c_batch_stride;
  p.c_ms = pr.c_m_stride;
  p.c_ns = pr.c_n_stride;
  p.beta = pr.beta;
  const int64_t total = (int64_t)pr.batch * pr.m * pr.n;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), (int64_t)ctx->sm_count * 8));
  fill_kernel<<<grid, 256, 0, s>>>(p);
  record_launch(ctx, pr.beta == 0.0f ? "contract_zero" : "contract_scale");
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fill launch");
  return LC_OK;
}

}  // namespace lc

// ---- failure detection: a bounded wait that can only run out ------------------------------------
namespace {

// One warp waits on an mbarrier that nothing ever arrives on, through the same bounded wait the
// GEMM kernels use (here with a short limit): it gives up, raises the device error word and
// returns, so the host sees LC_ERR_DEVICE_TIMEOUT at its next lc_sync and the context stays
// usable.
__global__ void __launch_bounds__(32) wait_probe_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    lcd::mbar_init(&bar, 1);
    lcd::fence_mbar_init();
  }
  __syncwarp();
  lcd::mbar_wait(&bar, 0, err, limit_ns);
}

}  // namespace

extern "C" {

lc_status lc_debug_wait_probe(lc_context* ctx, void* stream, uint32_t limit_us) {
  using namespace lc;
  if (ctx == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null context");
  if (limit_us == 0 || limit_us > 4000000u) return fail(LC_ERR_INVALID_ARGUMENT, "wait probe limit must be 1 us .. 4 s");
  wait_probe_kernel<<<1, 32, 0, stream_of(ctx, stream)>>>(ctx->d_error, (uint64_t)limit_us * 1000ull);
  record_launch(ctx, "debug_wait_probe");
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "wait probe launch");
  return LC_OK;
}

}  // extern "C"
