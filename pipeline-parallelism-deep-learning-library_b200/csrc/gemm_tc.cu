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
#include <mutex>
#include <string>

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
  int32_t mode;     // 0: C = alpha*acc + beta*C (+relu) ; 1: raw f32 partial
  int32_t c_dtype;  // LC_F32 / LC_BF16 / LC_F16
  int32_t relu;
  int32_t vec_ok;   // C rows contiguous (c_ns == 1) and 16-byte aligned for every 32-column group
  void* c;
  int64_t c_off, c_bs, c_ms, c_ns;
  float alpha, beta;
  float* partial;
  int* err;
  int32_t epi;       // 0 standard, 1 ReLU-mask by aux, 2 fused SGD into aux (f32) / aux2 (bf16)
  const void* aux;
  void* aux2;
  float lr;
};

template <int BN, bool TF32X3>
struct Cfg {
  static constexpr int EPR = TF32X3 ? 32 : 64;             // elements per 128-byte row
  static constexpr int BK = EPR;                           // K per stage
  static constexpr int UMMA_K = TF32X3 ? 8 : 16;           // K per instruction (32 bytes)
  static constexpr int KSTEPS = BK / UMMA_K;               // 4
  static constexpr int A_BYTES = kBM * kRowBytes;          // 16 KiB
  static constexpr int B_BYTES = BN * kRowBytes;
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * (TF32X3 ? 2 : 1);
  static constexpr int STAGES = (TF32X3 ? 196608 : 196608) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int THREADS = TF32X3 ? 320 : 192;
  // k-tiles per accumulator hand-off: one per unit for 16-bit inputs; 2 (64 K values, 24 MMAs)
  // for 3xTF32, which bounds the truncation bias of the tensor core's f32 accumulation to
  // about 24 ulp-halves per chunk while the chunks themselves are summed round-to-nearest.
  static constexpr int KC = TF32X3 ? 2 : (1 << 30);
  static constexpr int BAR_BYTES = 8 * (3 * STAGES + 5) + 16;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static_assert(STAGES >= 2, "at least two stages");
};

__device__ __forceinline__ void unit_coords(const KParams& p, int32_t u, int32_t* b, int32_t* split, int32_t* tm,
                                            int32_t* tn) {
  const int32_t per = p.tiles_m * p.tiles_n;
  const int32_t bs = u / per;
  int32_t t = u - bs * per;
  *b = bs / p.splits;
  *split = bs - *b * p.splits;
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

__device__ __forceinline__ void store_c(const KParams& p, int64_t idx, float v) {
  if (p.c_dtype == LC_F32) static_cast<float*>(p.c)[idx] = v;
  else if (p.c_dtype == LC_BF16) static_cast<uint16_t*>(p.c)[idx] = f32_to_bf16_rne(v);
  else static_cast<uint16_t*>(p.c)[idx] = __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ float finish(const KParams& p, float acc, float cold) {
  float v = __fmul_rn(p.alpha, acc);
  if (p.beta != 0.0f) v = __fadd_rn(v, __fmul_rn(p.beta, cold));
  if (p.relu) v = v > 0.0f ? v : 0.0f;
  return v;
}

__device__ __forceinline__ bool mask_on(const KParams& p, int64_t idx) {
  const uint16_t h = static_cast<const uint16_t*>(p.aux)[idx];
  return __uint_as_float(((uint32_t)h) << 16) > 0.0f;
}

// One output element through the selected epilogue (scalar path and split-K reduce).
__device__ __forceinline__ void apply_store(const KParams& p, int64_t idx, float acc) {
  if (p.epi == 0) {
    const float cold = p.beta != 0.0f ? load_c(p, idx) : 0.0f;
    store_c(p, idx, finish(p, acc, cold));
  } else if (p.epi == 1) {
    store_c(p, idx, mask_on(p, idx) ? __fmul_rn(p.alpha, acc) : 0.0f);
  } else {
    float* master = static_cast<float*>(const_cast<void*>(p.aux));
    const float step = __fmul_rn(p.lr, __fmul_rn(p.alpha, acc));
    const float w = __fsub_rn(master[idx], step);
    master[idx] = w;
    static_cast<uint16_t*>(p.aux2)[idx] = f32_to_bf16_rne(w);
  }
}

// Epilogue for one 32-column group of one row held by this thread.
__device__ __forceinline__ void epilogue_group(const KParams& p, const uint32_t (&r)[32], int32_t b, int32_t split,
                                               int32_t m, int32_t n0) {
  if (m >= p.M) return;
  if (p.mode == 1) {
    float* dst = p.partial + (((int64_t)split * p.batch + b) * p.M + m) * (int64_t)p.N + n0;
    if (n0 + 32 <= p.N && (p.N % 4) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                          __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n0 + j < p.N) dst[j] = __uint_as_float(r[j]);
    }
    return;
  }
  const int64_t base = p.c_off + (int64_t)b * p.c_bs + (int64_t)m * p.c_ms;
  if (p.vec_ok && n0 + 32 <= p.N && p.epi == 2) {
    // fused SGD: 16-byte master loads/stores and 16-byte bf16 stores
    const int64_t at = base + (int64_t)n0;
    float* master = static_cast<float*>(const_cast<void*>(p.aux)) + at;
    uint16_t* wb = static_cast<uint16_t*>(p.aux2) + at;
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float4 w0 = *reinterpret_cast<const float4*>(master + j);
      float4 w1 = *reinterpret_cast<const float4*>(master + j + 4);
      float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint4 out;
      uint16_t* oo = reinterpret_cast<uint16_t*>(&out);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        w[e] = __fsub_rn(w[e], __fmul_rn(p.lr, __fmul_rn(p.alpha, __uint_as_float(r[j + e]))));
        oo[e] = f32_to_bf16_rne(w[e]);
      }
      *reinterpret_cast<float4*>(master + j) = make_float4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<float4*>(master + j + 4) = make_float4(w[4], w[5], w[6], w[7]);
      *reinterpret_cast<uint4*>(wb + j) = out;
    }
    return;
  }
  if (p.vec_ok && n0 + 32 <= p.N && p.epi == 0) {
    const int64_t at = base + (int64_t)n0;  // c_ns == 1
    if (p.c_dtype == LC_F32) {
      float* dst = static_cast<float*>(p.c) + at;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.beta != 0.0f) old = *reinterpret_cast<const float4*>(dst + j);
        float4 v = make_float4(finish(p, __uint_as_float(r[j]), old.x), finish(p, __uint_as_float(r[j + 1]), old.y),
                               finish(p, __uint_as_float(r[j + 2]), old.z), finish(p, __uint_as_float(r[j + 3]), old.w));
        *reinterpret_cast<float4*>(dst + j) = v;
      }
    } else {
      uint16_t* dst = static_cast<uint16_t*>(p.c) + at;
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 old = make_uint4(0, 0, 0, 0);
        if (p.beta != 0.0f) old = *reinterpret_cast<const uint4*>(dst + j);
        const uint16_t* oh = reinterpret_cast<const uint16_t*>(&old);
        uint4 out;
        uint16_t* oo = reinterpret_cast<uint16_t*>(&out);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          float cold = p.c_dtype == LC_BF16 ? __uint_as_float(((uint32_t)oh[e]) << 16)
                                            : __half2float(__ushort_as_half(oh[e]));
          float v = finish(p, __uint_as_float(r[j + e]), cold);
          oo[e] = p.c_dtype == LC_BF16 ? f32_to_bf16_rne(v) : __half_as_ushort(__float2half_rn(v));
        }
        *reinterpret_cast<uint4*>(dst + j) = out;
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; j++) {
    const int32_t n = n0 + j;
    if (n < p.N) apply_store(p, base + (int64_t)n * p.c_ns, __uint_as_float(r[j]));
  }
}

template <int BN, bool TF32X3>
__global__ void __launch_bounds__(Cfg<BN, TF32X3>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const KParams p) {
  using C = Cfg<BN, TF32X3>;
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      lcd::mbar_init(&full[s], 1);
      lcd::mbar_init(&empty[s], 1);
      lcd::mbar_init(&conv[s], 128);
    }
    for (int a = 0; a < 2; a++) {
      lcd::mbar_init(&tfull[a], 1);
      lcd::mbar_init(&tempty[a], 128);
    }
    lcd::mbar_init(drain, 1);
    lcd::fence_mbar_init();
  }
  if (warp == 1) {
    lcd::tmem_alloc(tmem_slot, C::TMEM_COLS);
    lcd::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    lcd::tma_prefetch_desc(&tma_a);
    lcd::tma_prefetch_desc(&tma_b);
  }
  lcd::tc_fence_before();
  __syncthreads();
  lcd::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  constexpr uint32_t kStageTx = C::A_BYTES + C::B_BYTES;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int s = 0;
      uint32_t ph = 0;
      uint32_t filled = 0, last_par = 0;  // bit s: stage s filled at least once / parity of its last fill
      bool ok = true;
      for (int32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        int32_t b, split, tm, tn;
        unit_coords(p, u, &b, &split, &tm, &tn);
        const int32_t kb = split * p.kt_per_split;
        const int32_t ke = min(kb + p.kt_per_split, p.k_tiles);
        for (int32_t kt = kb; kt < ke; kt++) {
          if (!lcd::mbar_wait(&empty[s], ph ^ 1u, p.err)) {
            ok = false;
            break;
          }
          lcd::mbar_arrive_expect_tx(&full[s], kStageTx);
          const int32_t k0 = kt * C::BK;
          if (!p.a_mn) {
            lcd::tma_load_3d(a_hi(s), &tma_a, &full[s], k0, tm * kBM, b);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / C::EPR; j++)
              lcd::tma_load_3d(a_hi(s) + j * (C::BK * kRowBytes), &tma_a, &full[s], tm * kBM + j * C::EPR, k0, b);
          }
          if (!p.b_mn) {
            lcd::tma_load_3d(b_hi(s), &tma_b, &full[s], k0, tn * BN, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / C::EPR; j++)
              lcd::tma_load_3d(b_hi(s) + j * (C::BK * kRowBytes), &tma_b, &full[s], tn * BN + j * C::EPR, k0, b);
          }
          filled |= 1u << s;
          last_par = (last_par & ~(1u << s)) | (ph << s);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // never leave a bulk copy in flight into shared memory that is about to be released
      for (int t = 0; t < C::STAGES; t++)
        if (filled & (1u << t)) lcd::mbar_wait(&full[t], (last_par >> t) & 1u, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      // The accumulator is handed to the epilogue every KC k-tiles (a "chunk"): once per unit for
      // 16-bit inputs, every kChunkTiles k-tiles for 3xTF32, whose long sums the epilogue then
      // adds with round-to-nearest (the tensor core's own f32 accumulation truncates).
      int s = 0;
      uint32_t ph = 0;
      int32_t h = 0;  // hand-offs so far
      bool ok = true;
      for (int32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
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
        if (!lcd::mbar_wait(&tempty[acc], ((h >> 1) & 1) ^ 1u, p.err)) {
          ok = false;
          break;
        }
        lcd::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int32_t kt = c0; kt < c1; kt++) {
          if (!lcd::mbar_wait(TF32X3 ? &conv[s] : &full[s], ph, p.err)) {
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
            } else {
              lcd::umma_f16(d_tmem, da, db, p.idesc, accum);
            }
          }
          lcd::umma_commit(&empty[s]);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        lcd::umma_commit(&tfull[acc]);
        }
      }
      // every MMA this thread issued has retired before TMEM is released
      lcd::umma_commit(drain);
      lcd::mbar_wait(drain, 0, p.err);
    }
  } else if (warp < 6) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    int32_t h = 0;
    bool ok = true;
    for (int32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      int32_t b, split, tm, tn;
      unit_coords(p, u, &b, &split, &tm, &tn);
      const int32_t m = tm * kBM + q * 32 + lane;
      const int32_t kb = split * p.kt_per_split;
      const int32_t ke = min(kb + p.kt_per_split, p.k_tiles);
      if constexpr (TF32X3) {
        // running sum of the chunk accumulators, round-to-nearest f32 adds
        float run[BN];
#pragma unroll
        for (int j = 0; j < BN; j++) run[j] = 0.0f;
        for (int32_t c0 = kb; c0 < ke; c0 += C::KC, h++) {
          const int acc = h & 1;
          if (!lcd::mbar_wait(&tfull[acc], (h >> 1) & 1, p.err)) {
            ok = false;
            break;
          }
          lcd::tc_fence_after();
#pragma unroll
          for (int g = 0; g < BN / 32; g++) {
            uint32_t r[32];
            lcd::tmem_ld_32x32b_x32(lane_base + acc * BN + g * 32, r);
            lcd::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; j++) run[g * 32 + j] = __fadd_rn(run[g * 32 + j], __uint_as_float(r[j]));
          }
          lcd::tc_fence_before();
          lcd::mbar_arrive(&tempty[acc]);
        }
        if (!ok) break;
#pragma unroll
        for (int g = 0; g < BN / 32; g++) {
          uint32_t r[32];
#pragma unroll
          for (int j = 0; j < 32; j++) r[j] = __float_as_uint(run[g * 32 + j]);
          if (tn * BN + g * 32 < p.N) epilogue_group(p, r, b, split, m, tn * BN + g * 32);
        }
      } else {
        (void)kb;
        (void)ke;
        const int acc = h & 1;
        if (!lcd::mbar_wait(&tfull[acc], (h >> 1) & 1, p.err)) break;
        lcd::tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          lcd::tmem_ld_32x32b_x32(lane_base + acc * BN + c0, r);
          lcd::tmem_ld_wait();
          if (tn * BN + c0 < p.N) epilogue_group(p, r, b, split, m, tn * BN + c0);
        }
        lcd::tc_fence_before();
        lcd::mbar_arrive(&tempty[acc]);
        h++;
      }
    }
  } else if constexpr (TF32X3) {
    // ---------------- 3xTF32 split ----------------
    const int ct = threadIdx.x - 192;  // 0..127
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
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
        uint4* hi = reinterpret_cast<uint4*>(a_hi(s));
        uint4* lo = reinterpret_cast<uint4*>(a_lo(s));
        constexpr int NV = (C::A_BYTES + C::B_BYTES) / 16;
        for (int v = ct; v < NV; v += 128) {
          uint4 x = hi[v];
          uint4 h, l;
          const uint32_t* xs = reinterpret_cast<const uint32_t*>(&x);
          uint32_t* hs = reinterpret_cast<uint32_t*>(&h);
          uint32_t* ls = reinterpret_cast<uint32_t*>(&l);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            // hi = x rounded to tf32 (11 significant bits, nearest, ties away); lo = x - hi is
            // exact in f32 and is itself rounded to tf32 the same way, so the tensor core reads
            // both exactly whatever its own conversion does.
            uint32_t hb = (xs[e] + 0x1000u) & 0xffffe000u;
            if (((hb >> 23) & 0xffu) == 0xffu && ((xs[e] >> 23) & 0xffu) != 0xffu) hb = xs[e] & 0xffffe000u;
            const float hf = __uint_as_float(hb);
            hs[e] = hb;
            // an infinite or NaN hi carries the value alone (its lo would be NaN)
            const uint32_t lb = __float_as_uint(__fsub_rn(__uint_as_float(xs[e]), hf));
            ls[e] = isfinite(hf) ? ((lb + 0x1000u) & 0xffffe000u) : 0u;
          }
          hi[v] = h;
          lo[v] = l;
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

  __syncthreads();
  if (warp == 1) {
    lcd::tc_fence_after();
    lcd::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- split-K reduce: C = alpha * sum_s partial[s] + beta * C, splits summed in order -------------
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ partial, KParams p) {
  const int64_t per = (int64_t)p.M * p.N;
  const int64_t total = per * p.batch;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    float acc = 0.0f;
    for (int s = 0; s < p.splits; s++) acc = __fadd_rn(acc, partial[(int64_t)s * total + i]);
    const int64_t b = i / per;
    const int64_t rem = i - b * per;
    const int64_t m = rem / p.N, n = rem - (rem / p.N) * p.N;
    apply_store(p, p.c_off + b * p.c_bs + m * p.c_ms + n * p.c_ns, acc);
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

// 3-D map over (packed axis, row axis, batch) with a 128-byte-swizzled box of box_inner x box_rows.
// `atom32` selects the 32-byte-atom variant of the 128-byte swizzle (MN-major f32 tiles).
lc_status make_map(CUtensorMap* map, const void* base, int in_dtype, uint64_t inner, uint64_t rows,
                   uint64_t batch, uint64_t row_stride_b, uint64_t batch_stride_b, uint32_t box_inner,
                   uint32_t box_rows, bool atom32 = false) {
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
  return LC_OK;
}

template <int BN, bool TF32X3>
lc_status launch_kernel(lc_context* ctx, cudaStream_t s, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& p,
                        int grid) {
  using C = Cfg<BN, TF32X3>;
  static bool attr_set[64] = {false};
  auto kern = gemm_tc_kernel<BN, TF32X3>;
  if (!attr_set[ctx->device % 64]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return lc::cuda_fail(e, "cudaFuncSetAttribute(gemm)");
    attr_set[ctx->device % 64] = true;
  }
  kern<<<grid, C::THREADS, C::SMEM, s>>>(ta, tb, p);
  lc::record_launch(ctx, TF32X3 ? (BN == 64 ? "gemm_tf32x3_n64" : "gemm_tf32x3_n128")
                                : (BN == 64 ? "gemm_bf16_n64" : BN == 128 ? "gemm_bf16_n128" : "gemm_bf16_n256"));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return lc::cuda_fail(e, "gemm launch");
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

lc_status gemm_run(lc_context* ctx, cudaStream_t s, const GemmProblem& pr, lc_contract_plan* plan, bool dry_run) {
  GemmOperand A = pr.a, B = pr.b;
  uint64_t M = pr.m, N = pr.n;
  int64_t c_ms = pr.c_m_stride, c_ns = pr.c_n_stride;
  bool swap = false;
  // Skinny M: compute C^T = B^T A^T so the long side fills the 128-row MMA.
  if (M < 128 && N > M) {
    std::swap(A, B);
    std::swap(M, N);
    std::swap(c_ms, c_ns);
    swap = true;
  }
  const bool tf32x3 = pr.in_dtype == LC_F32;
  const int epr = tf32x3 ? 32 : 64;
  const size_t es = dtype_size(pr.in_dtype);
  int bn = N <= 64 ? 64 : (N <= 128 || tf32x3) ? 128 : 256;
  const int64_t tiles_m = ceil_div(M, 128), tiles_n = ceil_div(N, bn);
  const int64_t k_tiles = ceil_div(pr.k, epr);
  const int64_t tiles = tiles_m * tiles_n * pr.batch;
  int64_t splits = 1, kps = k_tiles;
  if (pr.splits_hint > 0) {
    splits = std::min<int64_t>(pr.splits_hint, k_tiles);
  } else if (tiles < ctx->sm_count && k_tiles >= 8) {
    splits = std::min<int64_t>(ceil_div(ctx->sm_count, tiles), k_tiles / 4);
    splits = std::max<int64_t>(splits, 1);
  }
  kps = ceil_div(k_tiles, splits);
  splits = ceil_div(k_tiles, kps);
  const int64_t units = tiles * splits;
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

  CUtensorMap ta, tb;
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
    st = make_map(&tb, bbase, pr.in_dtype, B.k, B.mn, pr.batch, rs, bstride(B, rs * B.mn), epr, bn);
  } else {
    uint64_t rs = B.k > 1 ? B.k_stride * es : ((B.mn * es + 15) / 16) * 16;
    st = make_map(&tb, bbase, pr.in_dtype, B.mn, B.k, pr.batch, rs, bstride(B, rs * B.k), epr, epr, tf32x3);
  }
  if (st) return st;

  KParams p{};
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.k_tiles = (int32_t)k_tiles;
  p.kt_per_split = (int32_t)kps;
  p.splits = (int32_t)splits;
  p.batch = (int32_t)pr.batch;
  p.tiles_m = (int32_t)tiles_m;
  p.tiles_n = (int32_t)tiles_n;
  p.units = (int32_t)units;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  const uint32_t fmt = tf32x3 ? 2u : (pr.in_dtype == LC_BF16 ? 1u : 0u);
  p.idesc = lcd::make_idesc(fmt, 128, bn, a_mn, b_mn);
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
  p.epi = pr.epi;
  p.aux = pr.aux;
  p.aux2 = pr.aux2;
  p.lr = pr.lr;
  auto rows_aligned = [&](const void* base, size_t es) {
    return c_ns == 1 && ((reinterpret_cast<uintptr_t>(base) + pr.c_offset * es) % 16 == 0) &&
           ((c_ms * es) % 16 == 0 || M == 1) && ((pr.c_batch_stride * es) % 16 == 0 || pr.batch == 1);
  };
  if (pr.epi == 2)
    p.vec_ok = rows_aligned(pr.aux, 4) && rows_aligned(pr.aux2, 2) ? 1 : 0;
  else
    p.vec_ok = rows_aligned(pr.c, dtype_size(pr.c_dtype)) ? 1 : 0;
  float* partial = nullptr;
  if (splits > 1) {
    st = scratch_alloc(ctx, s, sizeof(float) * (size_t)splits * pr.batch * M * N, (void**)&partial);
    if (st) return st;
    p.mode = 1;
    p.partial = partial;
  }
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(units, ctx->sm_count - pr.reserve_sms));
  if (tf32x3) {
    st = bn == 64 ? launch_kernel<64, true>(ctx, s, ta, tb, p, grid) : launch_kernel<128, true>(ctx, s, ta, tb, p, grid);
  } else {
    st = bn == 64    ? launch_kernel<64, false>(ctx, s, ta, tb, p, grid)
         : bn == 128 ? launch_kernel<128, false>(ctx, s, ta, tb, p, grid)
                     : launch_kernel<256, false>(ctx, s, ta, tb, p, grid);
  }
  if (st == LC_OK && splits > 1) {
    KParams rp = p;
    rp.mode = 0;
    const int64_t total = (int64_t)pr.batch * M * N;
    const int rgrid = (int)std::min<int64_t>(ceil_div(total, 256), (int64_t)ctx->sm_count * 8);
    splitk_reduce_kernel<<<rgrid, 256, 0, s>>>(partial, rp);
    record_launch(ctx, "gemm_splitk_reduce");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) st = cuda_fail(e, "split-K reduce launch");
  }
  if (partial) scratch_free(partial, s);
  return st;
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
