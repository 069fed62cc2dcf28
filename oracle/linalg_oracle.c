/*
 * linalg_oracle.c -- CPU restatement of the reference's algorithms for the hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or calls this
 * file: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * legs use it, as the checker and as the timed CPU baseline.
 *
 * Every function states which reference file:line it restates (paths are relative to the
 * reference project root, aaronilyas/Pipeline-Parallelism-Deep-Learning-Library).  The
 * reference is Rust; this is a plain-C restatement of the same arithmetic, compiled with
 * -O2 -ffp-contract=off and no fast-math, so every `a * b + c` rounds twice exactly as the
 * Rust code does (Rust never contracts to FMA).
 *
 * Pinning: the restatement is checked against the reference's own golden vectors and
 * known-answer tests (the JSON fixtures under tests/golden and tests/test_oracle_golden.py).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#if defined(__FP_FAST_FMAF) && !defined(LINALG_ORACLE_ALLOW_FMA)
/* -ffp-contract=off keeps the compiler from fusing; an explicit fmaf appears only where the
 * reference itself calls `mul_add` (or_mag32). */
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------------------ */
/* bf16 / f16 conversions                                                                 */
/* ------------------------------------------------------------------------------------ */

/* crates/cpu/src/lib.rs:725-731 `f32_bits_to_bf16`: nearest-even, NaN keeps sign and top
 * payload and becomes quiet.  Also the `half` 2.7.1 `bf16::from_f32_const` rounding for
 * non-NaN inputs (pinned by crates/cpu/src/invariants.rs:557-570). */
uint16_t or_f32_to_bf16(float x) {
    uint32_t bits = f2u(x);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    uint32_t lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}

/* crates/cpu/src/lib.rs:713-716 / :503-533: bf16 widens exactly into the top half. */
float or_bf16_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }

/* `half` 2.7.1 `f16::from_f32_const` (used by crates/cpu/src/lib.rs:708-711): IEEE binary16
 * nearest-even with overflow to infinity and gradual underflow.  Restated from IEEE 754;
 * pinned by the f16 cases of crates/cpu/src/invariants.rs:557-640. NaN payloads unpinned. */
uint16_t or_f32_to_f16(float x) {
    uint32_t b = f2u(x);
    uint32_t sign = (b >> 16) & 0x8000u;
    uint32_t exp = (b >> 23) & 0xffu;
    uint32_t man = b & 0x7fffffu;
    if (exp == 0xff) {
        if (man) return (uint16_t)(sign | 0x7e00u | (man >> 13));
        return (uint16_t)(sign | 0x7c00u);
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign; /* rounds to zero (below half the smallest subnormal) */
        uint32_t m = man | 0x800000u;          /* 24-bit significand */
        uint32_t shift = (uint32_t)(14 - e);   /* keep 10+e bits */
        uint32_t half_v = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half_v & 1u))) half_v += 1;
        return (uint16_t)(sign | half_v);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* carry may reach inf: correct */
    return (uint16_t)h;
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        int e = -1;
        do { man <<= 1; e++; } while (!(man & 0x400u));
        man &= 0x3ffu;
        return u2f(sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13));
    }
    return u2f(sign | ((exp - 15 + 127) << 23) | (man << 13));
}

void or_convert_f32_to_bf16(const float* x, uint16_t* y, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) y[i] = or_f32_to_bf16(x[i]);
}
void or_convert_bf16_to_f32(const uint16_t* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) y[i] = or_bf16_to_f32(x[i]);
}

/* ------------------------------------------------------------------------------------ */
/* GEMM: crates/cpu/src/lib.rs:203-295 (`gemm`) and :664-691 (`accumulate`).              */
/*   acc = (beta == 0 ? 0 : beta * C[r][c]);                                              */
/*   if alpha != 0: for k in 0..K: acc += alpha * A[r][k] * B[k][c]   (left-associative)   */
/*   C[r][c] = acc                                                                        */
/* The loop below hoists `alpha * A[r][k]` out of the column loop; each element still sees  */
/* the same operations in the same order, so the bits equal the reference's.               */
/* dtype: 1 = f32, 2 = f16, 3 = bf16 (crates/core/src/lib.rs:4-34 tags).                  */
/* Strides are in elements; any of the three supported layouts is expressed by strides.  */
/* ------------------------------------------------------------------------------------ */

static inline float load_any(const void* p, uint64_t i, int dtype) {
    if (dtype == 1) return ((const float*)p)[i];
    if (dtype == 2) return or_f16_to_f32(((const uint16_t*)p)[i]);
    return or_bf16_to_f32(((const uint16_t*)p)[i]);
}
static inline void store_any(void* p, uint64_t i, int dtype, float v) {
    if (dtype == 1) ((float*)p)[i] = v;
    else if (dtype == 2) ((uint16_t*)p)[i] = or_f32_to_f16(v);
    else ((uint16_t*)p)[i] = or_f32_to_bf16(v);
}

/* Mixed-dtype form: each operand widens exactly to f32 on load and C rounds on store, the
 * same `accumulate` loop.  B is widened once into a dense row-major f32 copy (exact), so the
 * inner loop is a plain f32 multiply-then-add that vectorises across columns without changing
 * any element's operation order.  `threads` > 1 splits the rows across POSIX threads; every
 * row is computed by one thread in the same order, so the bits do not depend on `threads`. */
typedef struct {
    int adt, cdt;
    uint64_t r0, r1, n, k;
    float alpha, beta;
    const void* a;
    uint64_t a_rs, a_cs;
    const float* bw;
    void* c;
    uint64_t c_rs, c_cs;
    int failed;
} gemm_rows_job;

static void* gemm_rows(void* arg) {
    gemm_rows_job* j = (gemm_rows_job*)arg;
    float* acc = (float*)malloc((j->n ? j->n : 1) * sizeof(float));
    if (!acc) { j->failed = 1; return NULL; }
    for (uint64_t r = j->r0; r < j->r1; r++) {
        for (uint64_t col = 0; col < j->n; col++)
            acc[col] = (j->beta == 0.0f) ? 0.0f : j->beta * load_any(j->c, r * j->c_rs + col * j->c_cs, j->cdt);
        if (j->bw) {
            for (uint64_t kk = 0; kk < j->k; kk++) {
                float ta = j->alpha * load_any(j->a, r * j->a_rs + kk * j->a_cs, j->adt);
                const float* bp = j->bw + kk * j->n;
                for (uint64_t col = 0; col < j->n; col++) acc[col] += ta * bp[col];
            }
        }
        for (uint64_t col = 0; col < j->n; col++) store_any(j->c, r * j->c_rs + col * j->c_cs, j->cdt, acc[col]);
    }
    free(acc);
    return NULL;
}

int or_gemm3(int adt, int bdt, int cdt, uint64_t m, uint64_t n, uint64_t k, float alpha, float beta,
             const void* a, uint64_t a_rs, uint64_t a_cs,
             const void* b, uint64_t b_rs, uint64_t b_cs,
             void* c, uint64_t c_rs, uint64_t c_cs, int threads) {
    float* bw = NULL;
    if (alpha != 0.0f && k > 0 && n > 0) {
        bw = (float*)malloc(k * n * sizeof(float));
        if (!bw) return -1;
        for (uint64_t kk = 0; kk < k; kk++)
            for (uint64_t col = 0; col < n; col++) bw[kk * n + col] = load_any(b, kk * b_rs + col * b_cs, bdt);
    }
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    if ((uint64_t)threads > m) threads = m > 0 ? (int)m : 1;
    gemm_rows_job jobs[64];
    pthread_t tids[64];
    int started[64] = {0};
    uint64_t per = (m + (uint64_t)threads - 1) / (uint64_t)threads;
    for (int t = 0; t < threads; t++) {
        uint64_t r0 = (uint64_t)t * per, r1 = r0 + per;
        if (r0 > m) r0 = m;
        if (r1 > m) r1 = m;
        gemm_rows_job j = {adt, cdt, r0, r1, n, k, alpha, beta, a, a_rs, a_cs, bw, c, c_rs, c_cs, 0};
        jobs[t] = j;
    }
    for (int t = 1; t < threads; t++) started[t] = pthread_create(&tids[t], NULL, gemm_rows, &jobs[t]) == 0;
    gemm_rows(&jobs[0]);
    int failed = jobs[0].failed;
    for (int t = 1; t < threads; t++) {
        if (started[t]) pthread_join(tids[t], NULL);
        else gemm_rows(&jobs[t]);
        failed |= jobs[t].failed;
    }
    free(bw);
    return failed ? -1 : 0;
}

int or_gemm(int dtype, uint64_t m, uint64_t n, uint64_t k, float alpha, float beta,
            const void* a, uint64_t a_rs, uint64_t a_cs,
            const void* b, uint64_t b_rs, uint64_t b_cs,
            void* c, uint64_t c_rs, uint64_t c_cs) {
    return or_gemm3(dtype, dtype, dtype, m, n, k, alpha, beta, a, a_rs, a_cs, b, b_rs, b_cs, c, c_rs,
                    c_cs, 1);
}

/* Same as or_gemm, but only the listed (row, col) entries are computed (used to time or
 * spot-check huge products the way tests/contraction_test.rs:1204-1227 samples entries).
 * out[i] receives the f32 accumulator of entry (rows[i], cols[i]) with beta = 0. */
void or_gemm_entries(int dtype, uint64_t k, float alpha,
                     const void* a, uint64_t a_rs, uint64_t a_cs,
                     const void* b, uint64_t b_rs, uint64_t b_cs,
                     const uint64_t* rows, const uint64_t* cols, uint64_t count, float* out) {
    for (uint64_t i = 0; i < count; i++) {
        float acc = 0.0f;
        if (alpha != 0.0f)
            for (uint64_t kk = 0; kk < k; kk++)
                acc += alpha * load_any(a, rows[i] * a_rs + kk * a_cs, dtype) *
                       load_any(b, kk * b_rs + cols[i] * b_cs, dtype);
        out[i] = acc;
    }
}

/* ------------------------------------------------------------------------------------ */
/* Contraction f64 reference: tests/contraction_test.rs:224-262 (`reference`).            */
/* For each output i: sum over contracted offsets in f64, |product| summed for the gate;  */
/* alpha scales both, beta*C0 added afterwards.  Offset tables are built by the caller    */
/* exactly as `offset_table` (:202-222) does.                                             */
/* ------------------------------------------------------------------------------------ */
void or_contract_f64(uint64_t n_out, uint64_t n_sum, double alpha, double beta,
                     const double* a, uint64_t a_off, const uint64_t* a_free, const uint64_t* a_sum,
                     const double* b, uint64_t b_off, const uint64_t* b_free, const uint64_t* b_sum,
                     const double* c0, const uint64_t* c_index,
                     double* exact, double* magnitude) {
    for (uint64_t i = 0; i < n_out; i++) {
        double sum = 0.0, mag = 0.0;
        if (alpha != 0.0) {
            uint64_t a0 = a_off + a_free[i], b0 = b_off + b_free[i];
            for (uint64_t s = 0; s < n_sum; s++) {
                double p = a[a0 + a_sum[s]] * b[b0 + b_sum[s]];
                sum += p;
                mag += fabs(p);
            }
            sum *= alpha;
            mag *= fabs(alpha);
        }
        if (beta != 0.0) {
            double t = beta * c0[c_index[i]];
            sum += t;
            mag += fabs(t);
        }
        exact[i] = sum;
        magnitude[i] = mag;
    }
}

/* ------------------------------------------------------------------------------------ */
/* Strided gather of raw words: tests/permutation_test.rs:85-117 (`gather_words`) and the  */
/* logical-element copy of tests/slicing_test.rs:163-250 (`logical_bytes`).               */
/* Element i of the row-major destination comes from src[offset + sum(idx[d]*stride[d])]. */
/* ------------------------------------------------------------------------------------ */
void or_gather(const uint8_t* src, uint64_t elem_bytes, uint64_t offset, int rank,
               const uint64_t* shape, const uint64_t* strides, uint8_t* dst) {
    uint64_t count = 1;
    for (int d = 0; d < rank; d++) count *= shape[d];
    uint64_t idx[8] = {0};
    for (uint64_t i = 0; i < count; i++) {
        uint64_t off = offset;
        for (int d = 0; d < rank; d++) off += idx[d] * strides[d];
        memcpy(dst + i * elem_bytes, src + off * elem_bytes, elem_bytes);
        for (int d = rank - 1; d >= 0; d--) {
            if (++idx[d] < shape[d]) break;
            idx[d] = 0;
        }
    }
}

/* Scatter counterpart (pack into a strided destination): element i of the logical order
 * goes to dst[offset + sum(idx*strides)]; src is logical row-major. */
void or_scatter(const uint8_t* src, uint64_t elem_bytes, uint8_t* dst, uint64_t offset, int rank,
                const uint64_t* shape, const uint64_t* strides) {
    uint64_t count = 1;
    for (int d = 0; d < rank; d++) count *= shape[d];
    uint64_t idx[8] = {0};
    for (uint64_t i = 0; i < count; i++) {
        uint64_t off = offset;
        for (int d = 0; d < rank; d++) off += idx[d] * strides[d];
        memcpy(dst + off * elem_bytes, src + i * elem_bytes, elem_bytes);
        for (int d = rank - 1; d >= 0; d--) {
            if (++idx[d] < shape[d]) break;
            idx[d] = 0;
        }
    }
}

/* ------------------------------------------------------------------------------------ */
/* Argmax of |x|: tests/argmax_test.rs:27-52 (`beats`, `ref_best`, `ref_argmax`).         */
/* NaN outranks every number (lowest NaN index wins); larger |x| wins; ties -> lowest.    */
/* Batched form: one answer per row of `cols` elements (row stride `row_stride`).         */
/* ------------------------------------------------------------------------------------ */
static inline int or_beats(float ma, uint64_t ia, float mb, uint64_t ib) {
    int na = isnan(ma), nb = isnan(mb);
    if (na && !nb) return 1;
    if (!na && nb) return 0;
    if (na && nb) return ia < ib;
    return ma > mb || (ma == mb && ia < ib);
}

uint64_t or_argmax(const float* x, uint64_t n, uint64_t stride) {
    float bm = 0.0f;
    uint64_t bi = 0;
    int have = 0;
    for (uint64_t i = 0; i < n; i++) {
        float m = fabsf(x[i * stride]);
        if (!have || or_beats(m, i, bm, bi)) { bm = m; bi = i; have = 1; }
    }
    return bi;
}

void or_argmax_rows(const float* x, uint64_t rows, uint64_t cols, uint64_t row_stride,
                    uint64_t col_stride, uint32_t* out) {
    for (uint64_t r = 0; r < rows; r++) out[r] = (uint32_t)or_argmax(x + r * row_stride, cols, col_stride);
}

/* Complex magnitude in f32: tests/argmax_test.rs:51-72 (`mag32`).  kind 0 = L1 (|re| + |im|),
 * kind 1 = Hypot (hi * sqrt(fma(r, r, 1)) with r = lo / hi, so nothing overflows near f32 max).
 * A NaN part gives NaN; subnormals take part (no flush to zero). */
float or_mag32(float re_in, float im_in, int kind) {
    float re = fabsf(re_in), im = fabsf(im_in);
    if (isnan(re) || isnan(im)) return NAN;
    if (kind == 0) return re + im;
    float hi = re > im ? re : im, lo = re > im ? im : re;
    if (hi == 0.0f) return 0.0f;
    if (isinf(hi)) return INFINITY;
    float r = lo / hi;
    return hi * sqrtf(fmaf(r, r, 1.0f));
}

/* `ref_argmax_complex` (tests/argmax_test.rs:74-76): `ref_best` over the f32 magnitudes of n
 * complex values (interleaved re, im) at a stride of `stride` complex elements. */
uint64_t or_argmax_complex(const float* z, uint64_t n, uint64_t stride, int kind) {
    float bm = 0.0f;
    uint64_t bi = 0;
    int have = 0;
    for (uint64_t i = 0; i < n; i++) {
        float m = or_mag32(z[2 * i * stride], z[2 * i * stride + 1], kind);
        if (!have || or_beats(m, i, bm, bi)) { bm = m; bi = i; have = 1; }
    }
    return bi;
}

/* ------------------------------------------------------------------------------------ */
/* sqrt: tests/sqrt_test.rs:25-27 `reference(x) = (x as f64).sqrt() as f32`.             */
/* reciprocal: tests/reciprocal_test.rs:137-140 `reference_real(x) = (1.0 / x as f64) as f32`. */
/* ------------------------------------------------------------------------------------ */
void or_sqrt(const float* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) y[i] = (float)sqrt((double)x[i]);
}
void or_reciprocal(const float* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) y[i] = (float)(1.0 / (double)x[i]);
}

/* ------------------------------------------------------------------------------------ */
/* Complex reciprocal: src/ops/reciprocal.rs:17-31 (documented rules) and                 */
/* shaders/reciprocal.metal:141-330 (the algorithm).  Smith's method on "split" floats:   */
/* a value is a significand m with |m| in [1, 2) (or a signed zero) and an exponent e,    */
/* x = m * 2^e, so no intermediate overflows, underflows or is flushed; every product and */
/* sum of significands is one f32 rounding, every division is the correctly rounded real */
/* reciprocal times the dividend, and the result is packed into f32 once (a subnormal    */
/* result rounds the 24-bit significand right, nearest even).                            */
/* ------------------------------------------------------------------------------------ */
typedef struct { float m; int e; } split_f;

static inline float rcp_cr(float x) { return (float)(1.0 / (double)x); }

/* nonzero finite bits -> split float (:141-153) */
static split_f split_of(uint32_t bits) {
    uint32_t ex = (bits >> 23) & 0xffu, fr = bits & 0x007fffffu, sg = bits & 0x80000000u;
    split_f s;
    if (ex == 0u) {
        int lead = 0;                      /* leading zeros of the 23-bit fraction in 32 bits */
        while (lead < 32 && !(fr & (0x80000000u >> lead))) lead++;
        int sh = lead - 8;
        s.m = u2f(((fr << sh) & 0x007fffffu) | (127u << 23) | sg);
        s.e = -126 - sh;
    } else {
        s.m = u2f((bits & 0x807fffffu) | (127u << 23));
        s.e = (int)ex - 127;
    }
    return s;
}

static split_f split_mul(split_f a, split_f b) {           /* :207-218 */
    split_f r;
    if (a.m == 0.0f || b.m == 0.0f) { r.m = a.m * b.m; r.e = 0; return r; }
    float p = a.m * b.m;
    if (fabsf(p) >= 2.0f) { r.m = p * 0.5f; r.e = a.e + b.e + 1; }
    else { r.m = p; r.e = a.e + b.e; }
    return r;
}

static split_f split_rcp(split_f a) {                      /* :220-227 */
    split_f r;
    float inv = rcp_cr(a.m);
    if (fabsf(inv) < 1.0f) { r.m = inv * 2.0f; r.e = -a.e - 1; }
    else { r.m = inv; r.e = -a.e; }
    return r;
}

static split_f split_add_same_sign(split_f a, split_f b) { /* :233-256 */
    if (b.m == 0.0f) return a;
    if (a.m == 0.0f) return b;
    if (a.e < b.e) { split_f t = a; a = b; b = t; }
    int diff = a.e - b.e;
    if (diff >= 25) return a;
    float s = a.m + b.m * u2f((uint32_t)(127 - diff) << 23);
    split_f r;
    if (fabsf(s) >= 2.0f) { r.m = s * 0.5f; r.e = a.e + 1; }
    else { r.m = s; r.e = a.e; }
    return r;
}

static int split_abs_ge(split_f a, split_f b) {            /* :258-271 */
    int az = a.m == 0.0f, bz = b.m == 0.0f;
    if (az) return bz;
    if (bz) return 1;
    if (a.e != b.e) return a.e > b.e;
    return fabsf(a.m) >= fabsf(b.m);
}

static uint32_t split_bits(split_f s) {                    /* :171-201 */
    uint32_t raw = f2u(s.m), sign = raw & 0x80000000u;
    if ((raw & 0x7fffffffu) == 0u) return sign;
    if (s.e >= 128) return sign | 0x7f800000u;
    if (s.e >= -126) return (raw & 0x807fffffu) | ((uint32_t)(s.e + 127) << 23);
    uint32_t rshift = (uint32_t)(-s.e - 126);
    uint32_t mant = (raw & 0x007fffffu) | 0x00800000u;
    uint32_t m;
    if (rshift >= 25u) {
        m = 0u;
    } else {
        uint32_t kept = mant >> rshift, rem = mant & ((1u << rshift) - 1u), half = 1u << (rshift - 1u);
        m = (rem > half || (rem == half && (kept & 1u))) ? kept + 1u : kept;
    }
    if (m == 0u) return sign;
    return sign | m;  /* m <= 2^23: a subnormal, or the carry into the smallest normal */
}

static split_f split_neg(split_f a) { a.m = -a.m; return a; }

/* :285-330 */
void or_reciprocal_c32(const uint32_t* z, uint32_t* w, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) {
        uint32_t ab = z[2 * i], bb = z[2 * i + 1];
        uint32_t ae = (ab >> 23) & 0xffu, be = (bb >> 23) & 0xffu;
        int a_inf = ae == 0xffu && !(ab & 0x007fffffu), b_inf = be == 0xffu && !(bb & 0x007fffffu);
        int a_nan = ae == 0xffu && (ab & 0x007fffffu), b_nan = be == 0xffu && (bb & 0x007fffffu);
        uint32_t re, im;
        if (a_inf || b_inf) {
            re = ab & 0x80000000u;
            im = (bb ^ 0x80000000u) & 0x80000000u;
        } else if (a_nan || b_nan) {
            re = im = 0x7fc00000u;
        } else if (!(bb & 0x7fffffffu)) {
            re = f2u(rcp_cr(u2f(ab)));
            im = (bb ^ 0x80000000u) & 0x80000000u;
        } else if (!(ab & 0x7fffffffu)) {
            re = ab & 0x80000000u;
            im = f2u(rcp_cr(u2f(bb))) ^ 0x80000000u;
        } else {
            split_f sa = split_of(ab), sb = split_of(bb);
            if (split_abs_ge(sa, sb)) {
                split_f r = split_mul(sb, split_rcp(sa));
                split_f inv = split_rcp(split_add_same_sign(sa, split_mul(sb, r)));
                re = split_bits(inv);
                im = split_bits(split_mul(split_neg(r), inv));
            } else {
                split_f r = split_mul(sa, split_rcp(sb));
                split_f inv = split_rcp(split_add_same_sign(sb, split_mul(sa, r)));
                re = split_bits(split_mul(r, inv));
                im = split_bits(split_neg(inv));
            }
        }
        w[2 * i] = re;
        w[2 * i + 1] = im;
    }
}

/* ------------------------------------------------------------------------------------ */
/* Training ops: crates/cpu/src/lib.rs:372-533 (sequential f32, no FMA).                  */
/* ------------------------------------------------------------------------------------ */

/* :372-401 add_bias: y[i][j] = x[i][j] + b[j]. */
void or_add_bias(const float* x, const float* b, float* y, uint64_t rows, uint64_t cols) {
    for (uint64_t r = 0; r < rows; r++)
        for (uint64_t c = 0; c < cols; c++) y[r * cols + c] = x[r * cols + c] + b[c];
}

/* :403-435 bias_grad: s[j] = sum over rows in order; db[j] = db[j] + s[j]. */
void or_bias_grad(const float* dpre, float* db, uint64_t rows, uint64_t cols) {
    if (rows == 0) return;
    for (uint64_t c = 0; c < cols; c++) {
        float s = 0.0f;
        for (uint64_t r = 0; r < rows; r++) s += dpre[r * cols + c];
        db[c] = db[c] + s;
    }
}

/* :437-472 mse_grad: d = y - t; sum += d*d; dy = (2*d)/n; loss = sum/n (n rounded to f32). */
float or_mse_grad(const float* y, const float* t, float* dy, uint64_t count) {
    float n = (float)count;
    float sum = 0.0f;
    for (uint64_t i = 0; i < count; i++) {
        float d = y[i] - t[i];
        sum += d * d;
        dy[i] = (2.0f * d) / n;
    }
    return sum / n;
}

/* :474-501 sgd_step: step = lr*dw; w = w - step; dw = +0. */
void or_sgd_step(float* w, float* dw, uint64_t count, float lr) {
    for (uint64_t i = 0; i < count; i++) {
        float step = lr * dw[i];
        w[i] = w[i] - step;
        dw[i] = 0.0f;
    }
}

/* ReLU is absent from the reference (the benchmark's MLP layers use it).  Stated as
 * `x > 0 ? x : +0`: -0, NaN and negatives give +0.  relu'(pre) selects dy where pre > 0.
 * The GPU kernels evaluate the same expression. */
void or_relu(const float* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}
void or_relu_backward(const float* pre, const float* dy, float* dx, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) dx[i] = pre[i] > 0.0f ? dy[i] : 0.0f;
}

/* :809-853 GELU with the Abramowitz-Stegun 7.1.26 erf, evaluated in f32. */
static const float ERF_A1 = 0.254829592f, ERF_A2 = 0.284496736f, ERF_A3 = 1.421413741f,
                   ERF_A4 = 1.453152027f, ERF_A5 = 1.061405429f, INV_SQRT_2PI = 0.3989422804014327f;
static float erf_f32(float x) {
    float sign = signbit(x) ? -1.0f : 1.0f;
    x = fabsf(x);
    float t = 1.0f / (1.0f + 0.3275911f * x);
    float poly = (((((ERF_A5 * t - ERF_A4) * t) + ERF_A3) * t - ERF_A2) * t + ERF_A1) * t;
    return sign * (1.0f - poly * expf(-x * x));
}
static const float FRAC_1_SQRT_2_F = 0.70710678118654752440f;
float or_gelu1(float x) { return 0.5f * x * (1.0f + erf_f32(x * FRAC_1_SQRT_2_F)); }
float or_gelu_prime1(float x) {
    float phi = 0.5f * (1.0f + erf_f32(x * FRAC_1_SQRT_2_F));
    float pdf = expf(-0.5f * x * x) * INV_SQRT_2PI;
    return phi + x * pdf;
}
void or_gelu(const float* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) y[i] = or_gelu1(x[i]);
}
void or_gelu_backward(const float* pre, const float* dy, float* dx, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) dx[i] = dy[i] * or_gelu_prime1(pre[i]);
}
uint32_t or_erf_constant_bits(int i) {
    const float v[6] = {ERF_A1, ERF_A2, ERF_A3, ERF_A4, ERF_A5, INV_SQRT_2PI};
    return f2u(v[i]);
}

/* ------------------------------------------------------------------------------------ */
/* Schedule and placement.                                                                */
/* crates/schedule/src/lib.rs:15-35 local_order; crates/pipeline/src/lib.rs:29-40.        */
/* ops[i] = +(m+1) for Forward(m), -(m+1) for Backward(m).  Returns count or -1.           */
/* ------------------------------------------------------------------------------------ */
int64_t or_local_order(uint64_t stages, uint64_t rank, uint64_t microbatches, int64_t* ops) {
    if (stages == 0 || rank >= stages || microbatches == 0 || microbatches > 0xffffffffull) return -1;
    uint64_t m = microbatches, w = stages - rank - 1;
    uint64_t warmup = w < m ? w : m;
    uint64_t steady = m - warmup;
    int64_t n = 0;
    for (uint64_t i = 0; i < warmup; i++) ops[n++] = (int64_t)i + 1;
    for (uint64_t i = 0; i < steady; i++) {
        ops[n++] = (int64_t)(warmup + i) + 1;
        ops[n++] = -((int64_t)i + 1);
    }
    for (uint64_t i = steady; i < m; i++) ops[n++] = -((int64_t)i + 1);
    return n;
}

int or_contiguous_placement(uint64_t layers, uint64_t stages, uint64_t* owners) {
    if (stages == 0 || layers == 0 || stages > layers) return -1;
    uint64_t base = layers / stages, extra = layers % stages, n = 0;
    for (uint64_t r = 0; r < stages; r++) {
        uint64_t count = base + (r < extra ? 1 : 0);
        for (uint64_t i = 0; i < count; i++) owners[n++] = r;
    }
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* Wire codec: crates/core/src/lib.rs:298-412 ("LNGL", version 1, dtype tag, ndim, u32    */
/* extents, little endian).  Returns header length or a negative error:                   */
/*   -1 = Error::Wire, -2 = Error::Shape.                                                  */
/* ------------------------------------------------------------------------------------ */
static uint64_t dtype_size_tag(uint32_t tag) { return tag == 1 ? 4 : (tag == 2 || tag == 3) ? 2 : 0; }

int64_t or_wire_write_header(uint32_t dtype_tag, const uint64_t* shape, uint32_t ndim, uint8_t* out,
                             uint64_t* payload_bytes) {
    if (ndim > 8) return -1;
    uint64_t numel = 1;
    for (uint32_t i = 0; i < ndim; i++) {
        if (shape[i] > 0xffffffffull) return -2;
        if (shape[i] != 0 && numel > UINT64_MAX / shape[i]) return -2;
        numel *= shape[i];
    }
    uint64_t sz = dtype_size_tag(dtype_tag);
    if (sz == 0) return -1;
    if (numel > UINT64_MAX / sz) return -2;
    *payload_bytes = numel * sz;
    const uint32_t words[4] = {0x4c474e4cu /* "LNGL" little endian */, 1u, dtype_tag, ndim};
    for (int i = 0; i < 4; i++)
        for (int b = 0; b < 4; b++) out[4 * i + b] = (uint8_t)(words[i] >> (8 * b));
    for (uint32_t i = 0; i < ndim; i++)
        for (int b = 0; b < 4; b++) out[16 + 4 * i + b] = (uint8_t)(shape[i] >> (8 * b));
    return 16 + 4 * (int64_t)ndim;
}

static uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* :361-389 parse_wire_header.  Returns payload offset (>= 16) or negative error. */
int64_t or_wire_parse_header(const uint8_t* bytes, uint64_t len, uint32_t* dtype_tag, uint64_t* shape,
                             uint32_t* ndim_out) {
    if (len < 16 || memcmp(bytes, "LNGL", 4) != 0) return -1;
    if (rd32(bytes + 4) != 1u) return -1;
    uint32_t tag = rd32(bytes + 8);
    if (dtype_size_tag(tag) == 0) return -1;
    uint32_t ndim = rd32(bytes + 12);
    if (ndim > 8) return -1;
    uint64_t header = 16 + 4 * (uint64_t)ndim;
    if (len < header) return -1;
    uint64_t numel = 1;
    for (uint32_t i = 0; i < ndim; i++) {
        uint64_t e = rd32(bytes + 16 + 4 * i);
        if (e != 0 && numel > UINT64_MAX / e) return -2;
        numel *= e;
        shape[i] = e;
    }
    uint64_t sz = dtype_size_tag(tag);
    if (numel > UINT64_MAX / sz) return -2;
    if (len - header != numel * sz) return -1;
    *dtype_tag = tag;
    *ndim_out = ndim;
    return (int64_t)header;
}

/* ------------------------------------------------------------------------------------ */
/* Pipeline reference: crates/pipeline/tests/pipeline.rs:396-480 (`reference`), the        */
/* sequential restatement of crates/pipeline/src/lib.rs:100-230 (`train`).                 */
/* Layers y = act(x @ W_l), W_l row-major [w[l], w[l+1]], f32; dy given per microbatch;    */
/* dW accumulated in microbatch order with beta = 1; dX = dpre @ W^T.                      */
/* act: 0 = GELU (crates/cpu/src/lib.rs:809-853), 1 = ReLU.                                 */
/* x: [mbs][batch][w0], dy: [mbs][batch][wL], y out: [mbs][batch][wL],                     */
/* dw out: concatenated per layer (zero-initialised by the caller).                        */
/* ------------------------------------------------------------------------------------ */
int or_train_reference(int act, uint64_t layers, const uint64_t* widths, uint64_t batch, uint64_t mbs,
                       const float* weights, const float* x, const float* dy, float* y, float* dw) {
    uint64_t maxw = 0, woff[65], total_w = 0;
    if (layers > 64) return -1;
    for (uint64_t l = 0; l <= layers; l++) if (widths[l] > maxw) maxw = widths[l];
    for (uint64_t l = 0; l < layers; l++) { woff[l] = total_w; total_w += widths[l] * widths[l + 1]; }
    float* acts = (float*)calloc((layers + 1) * batch * maxw, sizeof(float));
    float* pres = (float*)calloc(layers * batch * maxw, sizeof(float));
    float* g = (float*)calloc(batch * maxw, sizeof(float));
    float* dpre = (float*)calloc(batch * maxw, sizeof(float));
    float* dx = (float*)calloc(batch * maxw, sizeof(float));
    if (!acts || !pres || !g || !dpre || !dx) return -1;
    for (uint64_t mb = 0; mb < mbs; mb++) {
        memcpy(acts, x + mb * batch * widths[0], batch * widths[0] * sizeof(float));
        for (uint64_t l = 0; l < layers; l++) {
            uint64_t k = widths[l], n = widths[l + 1];
            float* a = acts + l * batch * maxw;
            float* pre = pres + l * batch * maxw;
            or_gemm(1, batch, n, k, 1.0f, 0.0f, a, k, 1, weights + woff[l], n, 1, pre, n, 1);
            float* out = acts + (l + 1) * batch * maxw;
            if (act == 0) or_gelu(pre, out, batch * n); else or_relu(pre, out, batch * n);
        }
        memcpy(y + mb * batch * widths[layers], acts + layers * batch * maxw,
               batch * widths[layers] * sizeof(float));
        memcpy(g, dy + mb * batch * widths[layers], batch * widths[layers] * sizeof(float));
        for (uint64_t l = layers; l-- > 0;) {
            uint64_t k = widths[l], n = widths[l + 1];
            float* pre = pres + l * batch * maxw;
            if (act == 0) or_gelu_backward(pre, g, dpre, batch * n); else or_relu_backward(pre, g, dpre, batch * n);
            float* in = acts + l * batch * maxw;
            /* dW[k, n] += in^T [k, batch] @ dpre [batch, n] */
            or_gemm(1, k, n, batch, 1.0f, 1.0f, in, 1, k, dpre, n, 1, dw + woff[l], n, 1);
            /* dX[batch, k] = dpre [batch, n] @ W^T [n, k] */
            or_gemm(1, batch, k, n, 1.0f, 0.0f, dpre, n, 1, weights + woff[l], 1, n, dx, k, 1);
            memcpy(g, dx, batch * k * sizeof(float));
        }
    }
    free(acts); free(pres); free(g); free(dpre); free(dx);
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* The benchmark training step (one optimizer step of the 1F1B MLP), stated with the       */
/* reference's Backend ops (crates/core/src/lib.rs:143-236, crates/cpu/src/lib.rs):        */
/*   weights: fp32 master W_l [d,d]; compute copy Wb_l = convert(W_l) to bf16.             */
/*   per microbatch m (rows m*mb .. m*mb+mb of X, T):                                      */
/*     h_0 = bf16(X_m);  h_{l+1} = bf16(relu(h_l @ Wb_l))  (f32 accumulate, one rounding)  */
/*     y = f32(h_L); d = y - T_m; dy = (2 d) / N with N = B*d (mean over the whole batch); */
/*     loss += sum d*d (f32, microbatch then element order); g = bf16(dy)                  */
/*     for l = L-1..0:  dpre = (h_{l+1} > 0) ? g : 0                                       */
/*                      dW_l += h_l^T @ dpre   (f32 accumulate into f32, beta = 1)         */
/*                      g = bf16(dpre @ Wb_l^T)                                            */
/*   loss /= N;  W_l = W_l - lr*dW_l;  dW_l = 0;  Wb_l = bf16(W_l)                         */
/* ReLU and the whole-batch MSE are this build's statement of the benchmark config; the   */
/* reference's own `train` uses GELU and a given dy (or_train_reference above).            */
/* x, t: [B][d] f32.  master: [L][d][d] f32 (updated in place).  Returns the loss.          */
/* ------------------------------------------------------------------------------------ */
float or_mlp_step(uint64_t layers, uint64_t d, uint64_t batch_total, uint64_t mb, float lr,
                  float* master, const float* x, const float* t, int threads) {
    uint64_t mbs = batch_total / mb;
    uint64_t dd = d * d;
    uint16_t* wb = (uint16_t*)malloc(layers * dd * sizeof(uint16_t));
    float* dw = (float*)calloc(layers * dd, sizeof(float));
    uint16_t* h = (uint16_t*)malloc((layers + 1) * mb * d * sizeof(uint16_t));
    float* pre = (float*)malloc(mb * d * sizeof(float));
    float* yd = (float*)malloc(mb * d * sizeof(float));
    uint16_t* g = (uint16_t*)malloc(mb * d * sizeof(uint16_t));
    uint16_t* dpre = (uint16_t*)malloc(mb * d * sizeof(uint16_t));
    if (!wb || !dw || !h || !pre || !yd || !g || !dpre) return NAN;
    for (uint64_t i = 0; i < layers * dd; i++) wb[i] = or_f32_to_bf16(master[i]);
    float n_total = (float)(batch_total * d);
    float loss = 0.0f;
    for (uint64_t m = 0; m < mbs; m++) {
        for (uint64_t i = 0; i < mb * d; i++) h[i] = or_f32_to_bf16(x[m * mb * d + i]);
        for (uint64_t l = 0; l < layers; l++) {
            or_gemm3(3, 3, 1, mb, d, d, 1.0f, 0.0f, h + l * mb * d, d, 1, wb + l * dd, d, 1, pre, d, 1, threads);
            uint16_t* out = h + (l + 1) * mb * d;
            for (uint64_t i = 0; i < mb * d; i++) out[i] = or_f32_to_bf16(pre[i] > 0.0f ? pre[i] : 0.0f);
        }
        const uint16_t* yb = h + layers * mb * d;
        for (uint64_t i = 0; i < mb * d; i++) {
            float dv = or_bf16_to_f32(yb[i]) - t[m * mb * d + i];
            loss += dv * dv;
            g[i] = or_f32_to_bf16((2.0f * dv) / n_total);
        }
        for (uint64_t l = layers; l-- > 0;) {
            const uint16_t* hin = h + l * mb * d;
            const uint16_t* hout = h + (l + 1) * mb * d;
            for (uint64_t i = 0; i < mb * d; i++) dpre[i] = or_bf16_to_f32(hout[i]) > 0.0f ? g[i] : 0;
            or_gemm3(3, 3, 1, d, d, mb, 1.0f, 1.0f, hin, 1, d, dpre, d, 1, dw + l * dd, d, 1, threads);
            or_gemm3(3, 3, 1, mb, d, d, 1.0f, 0.0f, dpre, d, 1, wb + l * dd, 1, d, yd, d, 1, threads);
            for (uint64_t i = 0; i < mb * d; i++) g[i] = or_f32_to_bf16(yd[i]);
        }
    }
    loss = loss / n_total;
    or_sgd_step(master, dw, layers * dd, lr);
    free(wb); free(dw); free(h); free(pre); free(yd); free(g); free(dpre);
    return loss;
}

/* ------------------------------------------------------------------------------------ */
/* f16 contraction of the op API: shaders/contraction.metal:445-702 (`two_sum`, `two_prod`, */
/* `dd_add`, `dd_mul`, `dd_to_half`, `store_dd`, `contract_general_f16`) and :733-755     */
/* (`contract_scale_f16`).  Each output: a double-float (hi, lo) sum of the exact f16 x f16 */
/* products in k order, times alpha, plus beta * C, rounded once to f16 (ties to even; an  */
/* f16 overflow of hi is kept).  Non-finite values take plain f32 arithmetic.             */
/* ------------------------------------------------------------------------------------ */
static void dd_two_sum(float a, float b, float* s, float* e) {
    *s = a + b;
    float v = *s - a;
    *e = (a - (*s - v)) + (b - v);
}
static void dd_two_prod(float a, float b, float* p, float* e) {
    *p = a * b;
    *e = fmaf(a, b, -*p);
}
static int fin3(float a, float b, float c) { return isfinite(a) && isfinite(b) && isfinite(c); }
static void dd_add1(float* hi, float* lo, float x) {
    if (!fin3(*hi, *lo, x)) { *hi = (*hi + x) + *lo; *lo = 0.0f; return; }
    float s, e;
    dd_two_sum(*hi, x, &s, &e);
    e = e + *lo;
    dd_two_sum(s, e, hi, lo);
}
static void dd_mul1(float* hi, float* lo, float s) {
    if (!fin3(*hi, *lo, s)) { *hi = fmaf(s, *hi, s * *lo); *lo = 0.0f; return; }
    float p1, e1, p2, e2;
    dd_two_prod(s, *hi, &p1, &e1);
    dd_two_prod(s, *lo, &p2, &e2);
    *hi = p1; *lo = e1;
    dd_add1(hi, lo, p2);
    dd_add1(hi, lo, e2);
}
static uint16_t f16_step1(uint16_t b, int up) {
    int neg = (b & 0x8000u) != 0;
    if (up != neg) return (uint16_t)(b + 1);
    if ((b & 0x7fffu) == 0) return up ? 0x0001 : 0x8001;
    return (uint16_t)(b - 1);
}
uint16_t or_dd_to_f16(float hi, float lo) {
    if (!isfinite(hi) || !isfinite(lo)) return or_f32_to_f16(hi + lo);
    uint16_t z = or_f32_to_f16(hi);
    if ((z & 0x7c00u) == 0x7c00u) return z;
    float zf = or_f16_to_f32(z);
    float r, rl;
    dd_two_sum(hi - zf, lo, &r, &rl);
    uint32_t mag = z & 0x7fffu;
    float ulp = mag < 0x0400u ? u2f(0x33800000u) : u2f((uint32_t)((int)(mag >> 10) - 25 + 127) << 23);
    uint32_t ex = (z >> 10) & 0x1fu;
    int pow2 = (z & 0x03ffu) == 0 && ex >= 2;
    float away = ulp * 0.5f, toward = pow2 ? ulp * 0.25f : away;
    int neg = (z & 0x8000u) != 0, odd = z & 1u;
    float up = neg ? toward : away, dn = neg ? away : toward;
    if (r > up || (r == up && (rl > 0.0f || (rl == 0.0f && odd)))) return f16_step1(z, 1);
    if (r < -dn || (r == -dn && (rl < 0.0f || (rl == 0.0f && odd)))) return f16_step1(z, 0);
    return z;
}

/* C[m x n] (f16 bits, row stride c_rs) = alpha * A B + beta * C; A element (i, k) at
 * a[i*a_rs + k*a_cs], B element (k, j) at b[k*b_rs + j*b_cs].  K = 0 or alpha = 0 with beta
 * != 0 is the once-rounded scale; beta == 0 with alpha == 0 writes +0. */
void or_contract_f16(uint64_t m, uint64_t n, uint64_t k, float alpha, float beta,
                     const uint16_t* a, uint64_t a_rs, uint64_t a_cs, const uint16_t* b, uint64_t b_rs,
                     uint64_t b_cs, uint16_t* c, uint64_t c_rs) {
    for (uint64_t i = 0; i < m; i++)
        for (uint64_t j = 0; j < n; j++) {
            uint16_t* cp = c + i * c_rs + j;
            if (alpha == 0.0f || k == 0) {
                if (beta == 0.0f) { *cp = 0; continue; }
                float cv = or_f16_to_f32(*cp), hi = 0.0f, lo = 0.0f;
                if (isfinite(beta) && isfinite(cv)) dd_two_prod(beta, cv, &hi, &lo);
                if (!isfinite(beta) || !isfinite(cv) || !isfinite(hi) || !isfinite(lo)) *cp = or_f32_to_f16(beta * cv);
                else *cp = or_dd_to_f16(hi, lo);
                continue;
            }
            float hi = 0.0f, lo = 0.0f;
            for (uint64_t kk = 0; kk < k; kk++)
                dd_add1(&hi, &lo, or_f16_to_f32(a[i * a_rs + kk * a_cs]) * or_f16_to_f32(b[kk * b_rs + j * b_cs]));
            dd_mul1(&hi, &lo, alpha);
            if (beta != 0.0f) {
                float cv = or_f16_to_f32(*cp);
                if (!fin3(hi, lo, cv)) { *cp = or_f32_to_f16((hi + lo) + beta * cv); continue; }
                float bh, bl;
                dd_two_prod(beta, cv, &bh, &bl);
                dd_add1(&hi, &lo, bh);
                dd_add1(&hi, &lo, bl);
            }
            *cp = or_dd_to_f16(hi, lo);
        }
}
