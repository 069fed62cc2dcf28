/*
 * linalg_b200.h -- C ABI of the B200 (sm_100a) implementation of the linalg hot path.
 *
 * This library replaces, behind plain C entry points, the reference project's op API
 * (the src/ops modules over src/abi.rs `TensorView`) and its `linalg_core::Backend` device slot
 * (crates/core/src/lib.rs:103-245, implemented today by crates/cpu, crates/metal and
 * crates/cuda), plus the 1F1B pipeline (crates/schedule, crates/pipeline) with NCCL
 * send/recv in place of crates/transport's byte messages.
 *
 * Conventions
 *  - Every function returns an `lc_status`; 0 is success.  On error nothing is launched and
 *    no output changes (src/abi.rs:20-22, crates/core/src/lib.rs:82, 88-96).  The message of
 *    the last error on the calling thread is `lc_last_error()`.
 *  - Device memory is owned by the caller.  A view never owns memory.  The library owns only
 *    its scratch (split-K partials, argmax candidates, operand staging), kept in a per-context
 *    stream-ordered pool.
 *  - `stream` is a `cudaStream_t` (NULL = the context's own stream).  Every `lc_encode_*`
 *    call is stream-ordered and returns before the device finishes; the plain form of each op
 *    enqueues on the context stream and waits, like the reference's sync wrappers.
 *  - Views: `data` is the buffer BASE (src/abi.rs:64-76), `offset`, `shape` and `strides`
 *    are in elements, strides are non-negative, `buffer_bytes` bounds every reachable element.
 */
#ifndef LINALG_B200_H
#define LINALG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LC_MAX_RANK 8
#define LC_MAX_CONCAT_PARTS 16

/* Status codes.  1..4 mirror `LinalgError` (src/abi.rs:24-33); 10..17 mirror
 * `linalg_core::Error` (crates/core/src/lib.rs:44-53). */
typedef int32_t lc_status;
enum {
    LC_OK = 0,
    LC_ERR_NO_DEVICE = 1,         /* LinalgError::NoDevice */
    LC_ERR_INVALID_ARGUMENT = 2,  /* LinalgError::InvalidArgument */
    LC_ERR_OVERLAP = 3,           /* LinalgError::Overlap */
    LC_ERR_LAUNCH = 4,            /* LinalgError::ShaderCompile: kernel could not be launched */
    LC_ERR_SHAPE = 10,            /* Error::Shape */
    LC_ERR_DTYPE = 11,            /* Error::Dtype */
    LC_ERR_UNSUPPORTED_LAYOUT = 12, /* Error::UnsupportedLayout */
    LC_ERR_UNSUPPORTED_DEVICE = 13, /* Error::UnsupportedDevice */
    LC_ERR_ALIAS = 14,            /* Error::Alias */
    LC_ERR_TRANSPORT = 15,        /* Error::Transport */
    LC_ERR_WIRE = 16,             /* Error::Wire */
    LC_ERR_SCHEDULE = 17,         /* Error::Schedule */
    LC_ERR_CUDA = 20,             /* a CUDA runtime call failed */
    LC_ERR_DEVICE_TIMEOUT = 21    /* a kernel's bounded wait ran out (device error flag set) */
};

/* Element types.  F32/F16/BF16 use crates/core/src/lib.rs:18-24's wire tags. */
typedef int32_t lc_dtype;
enum {
    LC_F32 = 1,
    LC_F16 = 2,
    LC_BF16 = 3,
    LC_U32 = 4,
    LC_I32 = 5,
    LC_C32 = 6, /* complex f32, (re, im) = [f32; 2] */
    LC_F64 = 7,
    LC_C64 = 8, /* 16-byte element (raw bits only) */
    LC_U16 = 9
};

/* Strided view: the reference's `TensorView<'a, T>` (src/abi.rs:64-76). */
typedef struct lc_view {
    void* data;             /* device address of the buffer base, never offset-adjusted */
    uint64_t buffer_bytes;  /* byte length of the buffer (`buffer.length()`) */
    uint64_t offset;        /* elements */
    int32_t dtype;          /* lc_dtype */
    int32_t rank;           /* 0..LC_MAX_RANK */
    uint64_t shape[LC_MAX_RANK];
    uint64_t strides[LC_MAX_RANK]; /* elements */
} lc_view;

typedef struct lc_context lc_context;

/* ---- context and memory --------------------------------------------------------------- */

/* Opens `device` and creates the context stream (replaces `MetalContext::new`,
 * src/abi.rs:55-61, and `CudaBackend::new`, crates/cuda/src/device.rs:150-234).
 * LC_ERR_NO_DEVICE when no CUDA device of compute capability 10.x is present. */
lc_status lc_context_create(int device, lc_context** out);
lc_status lc_context_destroy(lc_context* ctx);
/* The context's cudaStream_t. */
void* lc_context_stream(lc_context* ctx);
/* Waits for every launch on `stream` (NULL = context stream); then reports any device-side
 * bounded-wait timeout as LC_ERR_DEVICE_TIMEOUT (crates/core/src/lib.rs:136-141 `sync`). */
lc_status lc_sync(lc_context* ctx, void* stream);
/* Thread-local message of the last error (the String payload of LinalgError). */
const char* lc_last_error(void);
/* Number of kernel launches the library has issued on this context since creation
 * (`debug_launches().len()`, crates/core/src/lib.rs:238-244). */
uint64_t lc_debug_launches(lc_context* ctx);
/* Kernel name of launch `index` (0-based) for the most recent 4096 launches, or NULL. */
const char* lc_debug_launch_name(lc_context* ctx, uint64_t index);
/* Failure-detection probe (no reference counterpart): enqueues a one-warp kernel that waits,
 * through the bounded wait every library kernel uses, on a barrier nothing arrives on; after
 * `limit_us` (1 us .. 4 s) it gives up and raises the device error word, so the next lc_sync
 * returns LC_ERR_DEVICE_TIMEOUT and clears it.  No GPU fault, trap or hang is involved. */
lc_status lc_debug_wait_probe(lc_context* ctx, void* stream, uint32_t limit_us);

/* ---- views (host-only metadata; src/abi.rs:102-211, src/ops/permutation.rs:295-320,
 *      src/ops/slicing.rs:471-514) ------------------------------------------------------- */

/* `TensorView::validate` (src/abi.rs:145-177). */
lc_status lc_view_validate(const lc_view* v);
/* `permute_view` (src/ops/permutation.rs:299-320): axis i of out is axis perm[i] of v. */
lc_status lc_permute_view(const lc_view* v, const int32_t* perm, int32_t n, lc_view* out);
/* `slice` (src/ops/slicing.rs:478-514): one [start, end) range per axis. */
lc_status lc_slice(const lc_view* v, const uint64_t* starts, const uint64_t* ends, int32_t n, lc_view* out);

/* ---- contraction (src/ops/contraction.rs:1024-1130) --------------------------------------- */

/* C = alpha*A*B + beta*C over einsum labels (`encode_contract`, :1036-1048; `contract`,
 * :1053-1064).  f32 runs 3xTF32 on tcgen05 and bf16 kind::f16 with f32 accumulation; f16 rounds
 * each output once from a double-float dot, as the reference's op API does (:147-160, 829-836),
 * reading the operands in place whatever their strides. */
lc_status lc_encode_contract(lc_context* ctx, void* stream, float alpha, const lc_view* a,
                             const char* a_labels, const lc_view* b, const char* b_labels, float beta,
                             const lc_view* c, const char* c_labels);
lc_status lc_contract(lc_context* ctx, float alpha, const lc_view* a, const char* a_labels,
                      const lc_view* b, const char* b_labels, float beta, const lc_view* c,
                      const char* c_labels);
/* Batched matrix product over the leading rank-2 axes (`encode_gemm`, :1077-1088; `gemm`,
 * :1091-1102; `gemm_nowait`, :1116-1130 is `lc_encode_gemm` on the context stream). */
lc_status lc_encode_gemm(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b,
                         float beta, const lc_view* c);
lc_status lc_gemm(lc_context* ctx, float alpha, const lc_view* a, const lc_view* b, float beta,
                  const lc_view* c);
/* Fused epilogues: the training step's elementwise op applied by the product's own epilogue
 * warps, instead of a Backend::gemm followed by a separate training op (crates/core/src/lib.rs:
 * 166-236, the ops crates/pipeline/src/lib.rs:176-221 calls after each gemm; crates/cuda/train.cu
 * and gelu.cu are the reference's standalone kernels).  Every kind gives the bits of the unfused
 * sequence: the product rounded to f32 as lc_encode_gemm would store it, then the op.  `aux` and
 * `aux2` are views with C's shape, strides and offset. */
typedef enum lc_epilogue_kind {
    LC_EPI_NONE = 0,       /* C = alpha*A*B + beta*C (lc_encode_gemm) */
    LC_EPI_RELU = 1,       /* C = relu(alpha*A*B + beta*C): a ReLU layer's forward (the benchmark's
                              layers; the reference's own layers use `gelu`, :169) */
    LC_EPI_RELU_MASK = 2,  /* C = alpha*A*B where aux > 0, else +0; aux bf16 (16-bit inputs): the
                              data gradient through the ReLU of the layer whose input aux is
                              (lc_relu_backward's rule) */
    LC_EPI_SGD = 3,        /* C (f32 master weights) = C - lr*(alpha*A*B); aux2 (bf16) = bf16(C)
                              (16-bit inputs; beta unused): the weight gradient with `sgd_step`
                              and `convert` fused (crates/cpu/src/lib.rs:474-533) */
    LC_EPI_GELU = 4,       /* pre = alpha*A*B + beta*C; aux2 (optional) = pre; C = gelu(pre) (f32):
                              a layer's forward, `gemm` then `gelu` (crates/pipeline/src/lib.rs:
                              176-178; crates/cpu/src/lib.rs:809-853) */
    LC_EPI_GELU_BACKWARD = 5 /* C = gelu_backward(pre = aux, dy = alpha*A*B) (f32, beta 0): the data
                              gradient of layer l+1 fused with layer l's `gelu_backward` (:211, 220) */
} lc_epilogue_kind;
typedef struct lc_epilogue {
    int32_t kind;          /* lc_epilogue_kind */
    const lc_view* aux;
    const lc_view* aux2;
    float lr;
    /* plan hints, 0 = the planner's choice (the pipeline pins its grouped products with them) */
    int32_t tile_n;        /* kernel tile width 64, 128 or 256 (16-bit inputs) */
    int32_t splits;        /* split-K slices */
    int32_t swap;          /* 1: compute C^T = B^T A^T; -1: never */
} lc_epilogue;
lc_status lc_encode_gemm_fused(lc_context* ctx, void* stream, float alpha, const lc_view* a,
                               const lc_view* b, float beta, const lc_view* c,
                               const lc_epilogue* epi);
/* lc_encode_gemm that allocates no device memory (no counterpart in the reference, whose
 * backends allocate per call).  For callers that must not allocate while they run: a process
 * that reserves the card's memory up front, where a pool grown mid-step can run out, or a
 * latency-bound loop that a cudaMalloc/cudaFree or a pool growth would stall.  Same planning,
 * kernels and results as lc_encode_gemm, with the split-K scratch taken from fixed per-device
 * arrays: at most 16 MiB of partial sums (splits x batch x M x N f32) and 8192 tile counters,
 * which it zeroes on the stream before each split launch.  A product whose split does not fit,
 * or whose operands would need staging copies (no unit stride, or starts/strides not 16-byte
 * aligned), fails with LC_ERR_INVALID_ARGUMENT and launches nothing.  The arrays are shared by
 * every context, stream and thread of the process: calls whose kernels may overlap race and
 * give wrong results, so serialise them.  The first call on a device does set-up: it looks up
 * the arrays' device addresses, and under CUDA's default lazy module loading that lookup is what
 * loads the arrays onto the device (16 MiB + 32 KiB, held until the process exits).  Make that
 * first call before reserving the card's memory and before any stream capture. */
lc_status lc_encode_gemm_noalloc(lc_context* ctx, void* stream, float alpha, const lc_view* a,
                                 const lc_view* b, float beta, const lc_view* c);

/* Plan summary, for tests and reports (src/ops/contraction.rs:664-675 `Plan`). */
typedef struct lc_contract_plan {
    int32_t kind;    /* 0 Empty, 1 Fill, 2 Tiled, 3 Split, 4 Staged (operand materialised first),
                        5 General (f16: read in place, one rounding of a double-float dot) */
    int32_t splits;  /* split-K slices (1 when not split) */
    uint64_t batch, m, n, k;
    int32_t swap_ab; /* 1 when the kernel computes C^T = B^T A^T (skinny M) */
    int32_t a_major, b_major; /* 0 K-major, 1 MN-major, as fed to the tensor cores */
} lc_contract_plan;
lc_status lc_plan_contract(lc_context* ctx, float alpha, const lc_view* a, const char* a_labels,
                           const lc_view* b, const char* b_labels, float beta, const lc_view* c,
                           const char* c_labels, lc_contract_plan* out);

/* ---- permutation (src/ops/permutation.rs:322-387) ------------------------------------------ */

/* dst (row-major, same shape) = src (`materialize`, :326-342). */
lc_status lc_encode_materialize(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst);
lc_status lc_materialize(lc_context* ctx, const lc_view* src, const lc_view* dst);
/* dst = conj(src) (`conjugate`, :348-364); a plain copy for real element types. */
lc_status lc_encode_conjugate(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst);
/* dst = conj(src) with the last two axes swapped (`adjoint`, :371-387). */
lc_status lc_encode_adjoint(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst);

/* ---- slicing (src/ops/slicing.rs:516-753) -------------------------------------------------- */

/* dst = src elementwise, raw bits, 2/4/8/16-byte elements (`pack`, :519-585). */
lc_status lc_encode_pack(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst);
lc_status lc_pack(lc_context* ctx, const lc_view* src, const lc_view* dst);
/* Concatenate up to 16 parts along `axis` (`concat`, :589-753). */
lc_status lc_encode_concat(lc_context* ctx, void* stream, const lc_view* parts, int32_t n_parts,
                           int32_t axis, const lc_view* dst);

/* ---- argmax (src/ops/argmax.rs:80-213) ------------------------------------------------------ */

/* Index of the largest |x| of a rank-1 f32 view into a one-element u32 view (`encode_argmax`,
 * :96-103).  NaN outranks every number; ties go to the lowest index. */
lc_status lc_encode_argmax(lc_context* ctx, void* stream, const lc_view* x, const lc_view* out);
lc_status lc_argmax(lc_context* ctx, const lc_view* x, const lc_view* out);
/* Batched extension: argmax of |x| along the last axis for every leading index; `out` is a
 * u32 view of x's leading shape.  Same order as lc_encode_argmax per row. */
lc_status lc_encode_argmax_rows(lc_context* ctx, void* stream, const lc_view* x, const lc_view* out);
/* Complex magnitudes (`encode_argmax_complex`, :119-131): magnitude 0 = L1, 1 = Hypot. */
lc_status lc_encode_argmax_complex(lc_context* ctx, void* stream, const lc_view* x, int32_t magnitude,
                                   const lc_view* out);

/* ---- elementwise (src/ops/sqrt.rs:54-102, src/ops/reciprocal.rs:120-169) ------------------- */

/* Correctly rounded sqrt: bitwise (x as f64).sqrt() as f32.  In place when src == dst. */
lc_status lc_encode_sqrt(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst);
lc_status lc_sqrt(lc_context* ctx, const lc_view* src, const lc_view* dst);
/* 1/x.  Real f32: correctly rounded, bitwise (1.0 / x as f64) as f32.  Complex f32 (LC_C32):
 * Smith's algorithm on split floats with the C99 Annex G specials, bit for bit as the
 * reference kernel (src/ops/reciprocal.rs:17-31, shaders/reciprocal.metal:141-330). */
lc_status lc_encode_reciprocal(lc_context* ctx, void* stream, const lc_view* src, const lc_view* dst);
lc_status lc_reciprocal(lc_context* ctx, const lc_view* src, const lc_view* dst);

/* ---- Backend training ops (crates/core/src/lib.rs:143-236; crates/cuda/train.cu) ---------- */
/* Operands are row-major contiguous at offset 0 (else LC_ERR_UNSUPPORTED_LAYOUT); checks run
 * in the order Shape, Dtype, Alias, UnsupportedLayout (crates/core/src/lib.rs:88-96). */

/* `Backend::gemm` (crates/core/src/lib.rs:143-164): a [M,K], b [K,N], c [M,N], one dtype,
 * each row-major or (a or b) a `transpose_matrix` view; distinct buffers. */
lc_status lc_backend_gemm(lc_context* ctx, void* stream, const lc_view* a, const lc_view* b, const lc_view* c,
                          float alpha, float beta);
lc_status lc_add_bias(lc_context* ctx, void* stream, const lc_view* x, const lc_view* b, const lc_view* y);
lc_status lc_bias_grad(lc_context* ctx, void* stream, const lc_view* dpre, const lc_view* db);
/* Blocks until the loss is final (crates/core/src/lib.rs:203-217). */
lc_status lc_mse_grad(lc_context* ctx, void* stream, const lc_view* y, const lc_view* target, const lc_view* dy,
                      float* loss);
lc_status lc_sgd_step(lc_context* ctx, void* stream, const lc_view* w, const lc_view* dw, float lr);
lc_status lc_convert(lc_context* ctx, void* stream, const lc_view* x, const lc_view* y);
lc_status lc_gelu(lc_context* ctx, void* stream, const lc_view* x, const lc_view* y);
lc_status lc_gelu_backward(lc_context* ctx, void* stream, const lc_view* pre, const lc_view* dy, const lc_view* dx);
/* ReLU has no reference counterpart; the benchmark pipeline (Linear + ReLU) needs it. */
lc_status lc_relu(lc_context* ctx, void* stream, const lc_view* x, const lc_view* y);
lc_status lc_relu_backward(lc_context* ctx, void* stream, const lc_view* pre, const lc_view* dy, const lc_view* dx);

/* ---- schedule, placement and wire (host-only) ---------------------------------------------- */

/* `local_order` (crates/schedule/src/lib.rs:15-35): ops[i] = +(m+1) for Forward(m),
 * -(m+1) for Backward(m).  `capacity` >= 2*microbatches.  Writes the count to *count. */
lc_status lc_local_order(uint64_t stages, uint64_t rank, uint64_t microbatches, int64_t* ops,
                         uint64_t capacity, uint64_t* count);
/* `contiguous_placement` (crates/pipeline/src/lib.rs:29-40): owners[layer] = rank. */
lc_status lc_contiguous_placement(uint64_t layers, uint64_t stages, uint64_t* owners);
/* `write_wire_header` / `parse_wire_header` (crates/core/src/lib.rs:322-389). */
lc_status lc_wire_write_header(lc_dtype dtype, const uint64_t* shape, uint32_t ndim, uint8_t out[48],
                               uint64_t* header_len);
lc_status lc_wire_parse_header(const uint8_t* bytes, uint64_t len, lc_dtype* dtype, uint64_t shape[8],
                               uint32_t* ndim, uint64_t* payload_offset);

/* ---- host transports (crates/transport, the `Transport` trait crates/core/src/lib.rs:247-273) --
 * Byte messages between pipeline ranks that are host threads or processes (the GPU pipeline's
 * own data plane is NCCL).  Every failure is LC_ERR_TRANSPORT: a peer rank out of range or our
 * own, a timeout, a peer that is gone, a bad handshake.  Messages from one source arrive in order
 * and never merge with another source's.  A negative timeout waits forever. */
typedef struct lc_transport lc_transport;
/* `loopback(world)` (loopback.rs:21-28): `world` endpoints of one process in out[0..world). */
lc_status lc_transport_loopback(uint32_t world, lc_transport** out);
/* `localhost_mesh(world)` (tcp.rs:208-231): `world` endpoints connected over 127.0.0.1. */
lc_status lc_transport_localhost_mesh(uint32_t world, lc_transport** out);
/* `tcp_mesh_with_depth` (mesh.rs:38-87): this process's rank of a mesh whose rank r listens on
 * addrs[r] ("a.b.c.d:port"); dials lower ranks, accepts higher ones, LNGM handshake, within
 * `connect_timeout_ms`; `queue_depth` messages queue per peer before a send blocks (4 by default
 * in the reference). */
lc_status lc_transport_tcp_mesh(uint32_t rank, const char* const* addrs, uint32_t world,
                                int64_t connect_timeout_ms, uint32_t queue_depth, lc_transport** out);
/* Drops the endpoint: queued sends go out first, then the connections close. */
lc_status lc_transport_destroy(lc_transport* t);
uint32_t lc_transport_rank(const lc_transport* t);
uint32_t lc_transport_world(const lc_transport* t);
/* `send` / `send_parts` (core/src/lib.rs:252-262): one message, the concatenation of the parts;
 * returns once copied (blocks while the peer's queue is full). */
lc_status lc_transport_send(lc_transport* t, uint32_t dest, const void* bytes, uint64_t len);
lc_status lc_transport_send_parts(lc_transport* t, uint32_t dest, const void* const* parts,
                                  const uint64_t* lens, uint32_t n_parts);
/* `recv_timeout` (:254): the oldest message from `src`, in a buffer the caller releases with
 * lc_transport_free. */
lc_status lc_transport_recv(lc_transport* t, uint32_t src, int64_t timeout_ms, uint8_t** data,
                            uint64_t* len);
void lc_transport_free(uint8_t* data);
/* `send_tensor` / `recv_tensor` (crates/pipeline/src/lib.rs:71-98): a row-major device tensor
 * downloaded, framed with the LNGL header and sent; received, its dtype and shape checked against
 * `v` (LC_ERR_DTYPE / LC_ERR_SHAPE, LC_ERR_WIRE for a bad frame) and uploaded into it. */
lc_status lc_transport_send_tensor(lc_transport* t, uint32_t dest, lc_context* ctx, const lc_view* v);
lc_status lc_transport_recv_tensor(lc_transport* t, uint32_t src, int64_t timeout_ms, lc_context* ctx,
                                   const lc_view* v);

/* ---- 1F1B pipeline (crates/pipeline/src/lib.rs:100-230), one stage per GPU ---------------- */

typedef struct lc_pipeline lc_pipeline;

/* Two modes:
 *  - reference mode (compute_dtype LC_F32, loss 0, lr 0): exactly `train`'s dataflow with f32
 *    layers act(x @ W) (GELU or ReLU), dy supplied per microbatch, dW accumulated per
 *    microbatch with beta = 1 (read back with lc_pipeline_get_grad); any layer widths;
 *  - training mode (compute_dtype LC_BF16, activation ReLU, loss 1): the benchmark step: bf16
 *    compute weights with f32 master copies, MSE over the whole batch, SGD with `lr` fused into
 *    the weight-gradient GEMM (lr 0 keeps the gradient in lc_pipeline_get_grad instead). */
typedef struct lc_pipeline_config {
    uint64_t layers;        /* total layers across all stages */
    uint64_t width;         /* every layer is width x width when `widths` is NULL */
    const uint64_t* widths; /* optional: layers + 1 widths, layer l is widths[l] x widths[l+1] */
    uint64_t microbatch;    /* rows per microbatch */
    uint64_t microbatches;  /* microbatches per step */
    int32_t activation;     /* 0 = GELU (reference `train`), 1 = ReLU (benchmark) */
    int32_t compute_dtype;  /* LC_BF16 (fp32 master weights) or LC_F32 */
    float lr;               /* SGD learning rate (0 = no optimizer step) */
    int32_t loss;           /* 0 = dy supplied by the caller, 1 = MSE against targets */
    int32_t timeout_ms;     /* bound on every wait for a peer (crates/pipeline/src/lib.rs:19) */
} lc_pipeline_config;

/* Size of the opaque NCCL unique id that rank 0 creates and every rank receives. */
#define LC_PIPELINE_ID_BYTES 128
lc_status lc_pipeline_unique_id(uint8_t id[LC_PIPELINE_ID_BYTES]);
/* Creates stage `rank` of `world` on `device`; layers follow lc_contiguous_placement. */
lc_status lc_pipeline_create(const lc_pipeline_config* cfg, const uint8_t id[LC_PIPELINE_ID_BYTES], int32_t rank,
                             int32_t world, int32_t device, lc_pipeline** out);
lc_status lc_pipeline_destroy(lc_pipeline* p);
/* Layers this stage owns, in order: [first, first + count). */
lc_status lc_pipeline_local_layers(lc_pipeline* p, uint64_t* first, uint64_t* count);
/* Uploads fp32 master weights of local layer `index` (row-major, host memory). */
lc_status lc_pipeline_set_weight(lc_pipeline* p, uint64_t index, const float* host_w);
/* Fills every local layer with N(0, stddev^2) weights on the device, from a SplitMix64 stream
 * seeded with seed + global layer index (the same weights whatever the placement). */
lc_status lc_pipeline_init_weights(lc_pipeline* p, uint64_t seed, float stddev);
lc_status lc_pipeline_get_weight(lc_pipeline* p, uint64_t index, float* host_w);
/* Reads the f32 weight gradient accumulated by the last step (before the SGD zeroes it when
 * lr = 0, i.e. the reference `train` output dW). */
lc_status lc_pipeline_get_grad(lc_pipeline* p, uint64_t index, float* host_dw);
/* One training step.  Rank 0 passes inputs x [mbs*microbatch, width] f32 (host or device
 * pointer, `inputs_on_device`); the last rank passes targets (loss = 1) or dy (loss = 0).
 * Other ranks pass NULL.  The last rank's mean loss lands in *loss (others get 0).
 * The last rank may read the activations y of the last step with lc_pipeline_get_output. */
lc_status lc_pipeline_step(lc_pipeline* p, const float* x, const float* target_or_dy, int32_t inputs_on_device,
                           float* loss);
lc_status lc_pipeline_get_output(lc_pipeline* p, float* host_y);
/* Device time of the last step in milliseconds (CUDA events on the stage's compute stream). */
lc_status lc_pipeline_last_step_ms(lc_pipeline* p, float* ms);
/* Step trace (no reference counterpart; the reference's pipeline has no timing): with `on`,
 * every later step records CUDA events around each op's compute and each layer's weight update
 * (a few microseconds of event records per op).  lc_pipeline_trace then gives the last step's
 * records, 4 floats each: kind (1 forward, -1 backward, 2 weight update), first microbatch of
 * the op's group (or the global layer index of an update), start and end in ms from the step's
 * start.  `out` NULL: only *n is set; otherwise `cap` (records) must hold *n of them. */
lc_status lc_pipeline_set_trace(lc_pipeline* p, int32_t on);
lc_status lc_pipeline_trace(lc_pipeline* p, float* out, uint64_t cap, uint64_t* n);
/* The stage's compute stream (cudaStream_t); every step starts and ends on it. */
void* lc_pipeline_stream(lc_pipeline* p);
/* Kernel launches the stage has issued since creation (its `debug_launches().len()`). */
uint64_t lc_pipeline_debug_launches(lc_pipeline* p);

#ifdef __cplusplus
}
#endif
#endif /* LINALG_B200_H */
