// pipeline.cu -- 1F1B pipeline training, one stage per GPU, activations and gradients moved by
// NCCL send/recv over NVLink on dedicated streams (crates/pipeline/src/lib.rs:100-230 rebuilt).
//
// Streams per stage: the compute stream (all kernels), a forward-transfer stream and a
// backward-transfer stream.  Each transfer direction has its own communicator (the backward one
// is split from the forward one), so on each communicator a rank's operations form a one-way
// chain (forward: recv from r-1 then send to r+1, microbatch by microbatch) and can never wait on
// each other in a cycle.  CUDA events order compute against transfers; the compute stream never
// waits on a send, so sends behave like the reference's buffered transport.
//
// Training mode (the benchmark step; bf16 compute weights, f32 masters, ReLU, MSE, SGD):
//   forward  H[l+1] = relu(H[l] @ Wb_l)              one GEMM, ReLU fused in the epilogue
//   loss     dP[L-1] = bf16(2(y-t)/N) where y > 0    one kernel, deterministic partial sums
//   backward dP[l-1] = (dP[l] @ Wb_l^T) where H[l] > 0 one GEMM, ReLU' mask fused (H[l] is the
//            layer's stashed input); the mask for a stage's last layer is applied by the next
//            stage before it sends, so no mask crosses the link; rank 0 skips layer 0's dgrad
//   update   W_l -= lr * (H[l]^T @ dP[l]) over the whole batch (K = B), Wb_l = bf16(W_l), one
//            GEMM per layer with the SGD fused into its epilogue (no dW buffer at all)
// Reference mode (f32, GELU or ReLU, dy given): the reference's own dataflow with separate
// activation kernels and dW += x^T dpre per microbatch (beta = 1), exactly as `train` orders it.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "gemm.h"
#include "internal.h"

namespace {

using namespace lc;

// ---- NCCL, resolved at first use ---------------------------------------------------------------
// The library does not link libnccl: a process that already loaded NCCL (torch does) keeps its
// copy, and only a process without one loads libnccl.so.2 here.  Two copies of NCCL with the
// same soname in one process would otherwise race for the symbols at load time.
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommSplit)(ncclComm_t, int, int, ncclComm_t*, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) return;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    api.ok = sym(api.GetUniqueId, "ncclGetUniqueId") && sym(api.CommInitRankConfig, "ncclCommInitRankConfig") &&
             sym(api.CommSplit, "ncclCommSplit") && sym(api.CommDestroy, "ncclCommDestroy") &&
             sym(api.CommAbort, "ncclCommAbort") && sym(api.CommGetAsyncError, "ncclCommGetAsyncError") &&
             sym(api.Send, "ncclSend") && sym(api.Recv, "ncclRecv") && sym(api.GetErrorString, "ncclGetErrorString");
  });
  return api;
}

// ---- kernels ----------------------------------------------------------------------------------

__device__ __forceinline__ uint16_t bf16_bits(float x) {
  uint32_t bits = __float_as_uint(x);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
  uint32_t lsb = (bits >> 16) & 1u;
  return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}

__device__ __forceinline__ float bf16_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

__global__ void to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) y[i] = bf16_bits(x[i]);
}

// MSE over the whole batch with the ReLU' of the last layer folded in:
//   d = f32(y) - t;  part += d*d;  g = (y > 0) ? bf16((2*d)/N) : 0
constexpr int kMseThreads = 256;
constexpr int kMseBlocks = 296;  // 2 per SM: the loss gradient of one microbatch in one wave
// microbatches per product on a stage holding every layer: 32 x 8192 step on one B200, 55.4k
// samples/s with 4 (256-row products), 48.2k with 2, 32.2k with 1
constexpr uint64_t kFuseDefault = 4;
constexpr int kNcclCtas = 0;     // CTAs per NCCL transfer kernel (communicator maxCTAs); 0 = NCCL's choice
// dy = relu'(y) * (2 * (y - t)) / n and per-block partial sums of (y - t)^2, 8 elements at a time
// (16-byte loads of y and g, two of t); the partials are summed in a fixed order by
// loss_reduce_kernel, so the loss is deterministic.
__global__ void __launch_bounds__(kMseThreads) mse_relu_kernel(const uint16_t* __restrict__ y, const float* __restrict__ t,
                                                                uint16_t* __restrict__ g, uint64_t n, float n_total,
                                                                float* __restrict__ part) {
  __shared__ float red[kMseThreads];
  float acc = 0.0f;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  // 16-byte accesses only when all three arrays start 16-byte aligned (widths that are not a
  // multiple of 8 shift microbatch rows off alignment); otherwise the element loop below does it all
  const bool vec = ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(t)) &
                    15u) == 0;
  const uint64_t n8 = vec ? n / 8 : 0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
    const uint4 yr = __ldcs(reinterpret_cast<const uint4*>(y) + i);
    const float4 t0 = __ldcs(reinterpret_cast<const float4*>(t) + 2 * i);
    const float4 t1 = __ldcs(reinterpret_cast<const float4*>(t) + 2 * i + 1);
    const uint32_t yw[4] = {yr.x, yr.y, yr.z, yr.w};
    const float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
    uint32_t gw[4];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const float yv = bf16_f32((uint16_t)(e & 1 ? yw[e / 2] >> 16 : yw[e / 2] & 0xffffu));
      const float d = __fsub_rn(yv, tv[e]);
      acc = __fadd_rn(acc, __fmul_rn(d, d));
      const uint32_t gb = yv > 0.0f ? bf16_bits(__fdiv_rn(__fmul_rn(2.0f, d), n_total)) : 0u;
      if (e & 1) gw[e / 2] |= gb << 16;
      else gw[e / 2] = gb;
    }
    reinterpret_cast<uint4*>(g)[i] = make_uint4(gw[0], gw[1], gw[2], gw[3]);
  }
  for (uint64_t i = n8 * 8 + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float yv = bf16_f32(y[i]);
    const float d = __fsub_rn(yv, t[i]);
    acc = __fadd_rn(acc, __fmul_rn(d, d));
    g[i] = yv > 0.0f ? bf16_bits(__fdiv_rn(__fmul_rn(2.0f, d), n_total)) : (uint16_t)0;
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = kMseThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = red[0];
}

__global__ void __launch_bounds__(kMseThreads) loss_reduce_kernel(const float* __restrict__ part, int count, float n_total,
                                                                   float* __restrict__ loss) {
  __shared__ float red[kMseThreads];
  float acc = 0.0f;
  for (int i = threadIdx.x; i < count; i += kMseThreads) acc = __fadd_rn(acc, part[i]);
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = kMseThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = __fdiv_rn(red[0], n_total);
}

// N(0, stddev^2) from SplitMix64 draws 2i and 2i+1 of `seed` (Box-Muller, one rounding to f32).
__device__ __forceinline__ uint64_t splitmix(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void normal_init_kernel(float* __restrict__ w, uint16_t* __restrict__ wb, uint64_t n, uint64_t seed,
                                   float stddev) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const double u1 = ((double)(splitmix(seed, 2 * i) >> 11) + 1.0) * 0x1.0p-53;
    const double u2 = (double)(splitmix(seed, 2 * i + 1) >> 11) * 0x1.0p-53;
    const double z = sqrt(-2.0 * log(u1)) * cospi(2.0 * u2);
    const float v = (float)(z * (double)stddev);
    w[i] = v;
    if (wb) wb[i] = bf16_bits(v);
  }
}

unsigned blocks_for(lc_context* ctx, uint64_t n, unsigned per = 256) {
  uint64_t b = (n + per - 1) / per;
  uint64_t cap = (uint64_t)ctx->sm_count * 8;
  return (unsigned)std::max<uint64_t>(1, std::min(b, cap));
}

// ---- helpers -----------------------------------------------------------------------------------

lc_status nccl_fail(ncclResult_t r, const char* what) {
  const char* s = nccl().ok ? nccl().GetErrorString(r) : "NCCL unavailable";
  return fail(LC_ERR_TRANSPORT, std::string(what) + ": " + s);
}

#define CU(x)                                          \
  do {                                                 \
    cudaError_t e_ = (x);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #x);   \
  } while (0)
#define NC(x)                                          \
  do {                                                 \
    ncclResult_t r_ = (x);                             \
    if (r_ != ncclSuccess) return nccl_fail(r_, #x);   \
  } while (0)

lc_view matrix_view(void* data, int32_t dtype, uint64_t rows, uint64_t cols, uint64_t buffer_bytes) {
  lc_view v{};
  v.data = data;
  v.buffer_bytes = buffer_bytes;
  v.dtype = dtype;
  v.rank = 2;
  v.shape[0] = rows;
  v.shape[1] = cols;
  v.strides[0] = cols;
  v.strides[1] = 1;
  return v;
}

}  // namespace

struct lc_pipeline {
  lc_pipeline_config cfg{};
  std::vector<uint64_t> widths;  // global, layers + 1
  int rank = 0, world = 1, device = 0;
  bool train_mode = false;
  lc_context* ctx = nullptr;
  cudaStream_t s_fwd = nullptr, s_bwd = nullptr;
  // Training mode: extra compute streams.  In 1F1B the forwards of different microbatches are
  // independent, so are the backwards, and B(m) needs only F(m): forwards run on the even
  // streams (0 = the context stream), backwards on the odd ones, microbatch m on pair m % (K/2),
  // so K/2 forwards and K/2 backwards can share the GPU and hide each other's per-layer gaps.
  std::vector<cudaStream_t> s_work;  // streams 1 .. K-1 (K = kernels that may share the GPU)
  int n_streams = 1;
  ncclComm_t comm_fwd = nullptr, comm_bwd = nullptr;
  uint64_t first = 0, count = 0, B = 0;
  std::vector<float*> master, dw, pre;
  std::vector<void*> wb, H, dP;
  void* gsend = nullptr;       // backward send buffer (rank > 0)
  void* dbuf = nullptr;        // reference mode: per-microbatch dpre / dx scratch
  void* dbuf2 = nullptr;
  float* x_dev = nullptr;      // rank 0 input staging (f32 [B, w0])
  float* t_dev = nullptr;      // last rank targets or dy staging (f32 [B, wL])
  float* part = nullptr;       // loss partials
  float* loss_dev = nullptr;
  float* loss_host = nullptr;  // pinned
  cudaEvent_t ev_start = nullptr, ev_end = nullptr, ev_fwd_join = nullptr, ev_bwd_join = nullptr;
  cudaEvent_t ev_inputs = nullptr;          // the step's inputs are on the device
  std::vector<cudaEvent_t> ev_work_join;     // per extra compute stream: its last op of the step
  std::vector<cudaEvent_t> ev_fr, ev_fd, ev_br, ev_bd;
  std::vector<cudaEvent_t> ev_fdone;  // microbatch m's forward (and loss gradient) complete
  // One stage holding every layer (training mode): consecutive microbatches run in groups of
  // `fuse` as one product per layer, so one pass over a weight matrix serves the whole group.
  struct Shape {
    int32_t bn = 0, splits = 0, swap = 0;
  };
  uint64_t fuse = 0;  // 0 = not decided yet
  std::vector<Shape> fwd_shape, dgrad_shape;
  float last_ms = 0.0f;
  bool aborted = false;
  // Step trace (lc_pipeline_set_trace): timing events around every op's compute and around the
  // weight updates; after the step, one record per op of (kind, first microbatch, start, end) in
  // ms from the step start.  kind: 1 forward, -1 backward, 2 weight update of one layer.
  bool trace = false;
  std::vector<cudaEvent_t> ev_t0, ev_t1;
  std::vector<float> trace_rec;

  uint64_t win(uint64_t l) const { return widths[first + l]; }       // local layer l input width
  uint64_t wout(uint64_t l) const { return widths[first + l + 1]; }  // local layer l output width
  bool is_first() const { return rank == 0; }
  bool is_last() const { return rank + 1 == world; }
  cudaStream_t comp() const { return ctx->stream; }
  cudaStream_t work(int i) const { return i == 0 ? ctx->stream : s_work[i - 1]; }
  cudaStream_t fwd_stream(uint64_t m) const { return n_streams > 1 ? work((int)(2 * (m % (n_streams / 2)))) : ctx->stream; }
  cudaStream_t back_stream(uint64_t m) const {
    return n_streams > 1 ? work((int)(2 * (m % (n_streams / 2)) + 1)) : ctx->stream;
  }
  size_t es() const { return train_mode ? 2 : 4; }
};

namespace {

lc_status alloc(void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_fail(e, "pipeline cudaMalloc");
  return LC_OK;
}

// Host <-> device copy ordered on the stage's own (non-blocking) stream and waited for.  A plain
// cudaMemcpy runs on the legacy stream, which a non-blocking stream does not wait for, and from
// pageable memory it may return before its DMA has landed.
lc_status copy_sync(lc_pipeline* p, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind) {
  CU(cudaMemcpyAsync(dst, src, bytes, kind, p->comp()));
  CU(cudaStreamSynchronize(p->comp()));
  return LC_OK;
}

lc_status setup(lc_pipeline* p) {
  const uint64_t mbs = p->cfg.microbatches, mb = p->cfg.microbatch;
  p->B = mbs * mb;
  CU(cudaStreamCreateWithFlags(&p->s_fwd, cudaStreamNonBlocking));
  CU(cudaStreamCreateWithFlags(&p->s_bwd, cudaStreamNonBlocking));
  CU(cudaEventCreate(&p->ev_start));
  CU(cudaEventCreate(&p->ev_end));
  CU(cudaEventCreateWithFlags(&p->ev_fwd_join, cudaEventDisableTiming));
  CU(cudaEventCreateWithFlags(&p->ev_bwd_join, cudaEventDisableTiming));
  CU(cudaEventCreateWithFlags(&p->ev_inputs, cudaEventDisableTiming));
  if (p->train_mode) {
    static const int env_streams = [] {
      const char* e = getenv("LC_PIPE_STREAMS");  // tuning override: compute streams (1, 2, 4 or 8)
      return e ? atoi(e) : 0;
    }();
    // One stage holding every layer (N = 1) has all of 1F1B's independent forwards and backwards
    // to overlap: four streams.  With several stages the transfers gate the microbatches and about
    // two chains are ready at a time: two streams, each chain on half of the GPU (measured on 4
    // B200s: 103k samples/s with two streams, 66k with four, 90k with one).
    const int dflt = p->world > 1 ? 2 : 4;
    p->n_streams = env_streams == 1 || env_streams == 2 || env_streams == 4 || env_streams == 8 ? env_streams : dflt;
    p->s_work.resize(p->n_streams - 1);
    p->ev_work_join.resize(p->n_streams - 1);
    for (auto& q : p->s_work) CU(cudaStreamCreateWithFlags(&q, cudaStreamNonBlocking));
    for (auto& e : p->ev_work_join) CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  for (auto* v : {&p->ev_fr, &p->ev_fd, &p->ev_br, &p->ev_bd, &p->ev_fdone}) {
    v->resize(mbs);
    for (auto& e : *v) CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  const size_t es = p->es();
  lc_status st;
  for (uint64_t l = 0; l < p->count; l++) {
    const uint64_t n = p->win(l) * p->wout(l);
    float* m = nullptr;
    if ((st = alloc((void**)&m, n * 4))) return st;
    CU(cudaMemset(m, 0, n * 4));
    p->master.push_back(m);
    if (p->train_mode) {
      void* b = nullptr;
      if ((st = alloc(&b, n * 2))) return st;
      CU(cudaMemset(b, 0, n * 2));
      p->wb.push_back(b);
    }
    if (!p->train_mode || p->cfg.lr == 0.0f) {
      float* g = nullptr;
      if ((st = alloc((void**)&g, n * 4))) return st;
      CU(cudaMemset(g, 0, n * 4));
      p->dw.push_back(g);
    }
  }
  for (uint64_t l = 0; l <= p->count; l++) {
    void* h = nullptr;
    const uint64_t w = l < p->count ? p->win(l) : p->wout(p->count - 1);
    if ((st = alloc(&h, p->B * w * es))) return st;
    p->H.push_back(h);
  }
  for (uint64_t l = 0; l < p->count; l++) {
    if (p->train_mode) {
      void* d = nullptr;
      if ((st = alloc(&d, p->B * p->wout(l) * 2))) return st;
      p->dP.push_back(d);
    } else {
      float* q = nullptr;
      if ((st = alloc((void**)&q, p->B * p->wout(l) * 4))) return st;
      p->pre.push_back(q);
    }
  }
  if (!p->is_first() && (st = alloc(&p->gsend, p->B * p->win(0) * es))) return st;
  if (!p->train_mode) {
    uint64_t maxw = 0;
    for (uint64_t l = 0; l <= p->count; l++) maxw = std::max(maxw, p->widths[p->first + l]);
    if ((st = alloc(&p->dbuf, mb * maxw * 4))) return st;
    if ((st = alloc(&p->dbuf2, mb * maxw * 4))) return st;
    if (!p->is_last()) {  // received gradients (f32 [B, wL_local])
      void* g = nullptr;
      if ((st = alloc(&g, p->B * p->wout(p->count - 1) * 4))) return st;
      p->dP.push_back(g);
    }
  }
  if (p->is_first() && (st = alloc((void**)&p->x_dev, p->B * p->widths[0] * 4))) return st;
  if (p->is_last() && (st = alloc((void**)&p->t_dev, p->B * p->widths.back() * 4))) return st;
  if ((st = alloc((void**)&p->part, sizeof(float) * kMseBlocks * mbs))) return st;
  if ((st = alloc((void**)&p->loss_dev, sizeof(float)))) return st;
  CU(cudaMallocHost(&p->loss_host, sizeof(float)));
  // the zero fills above ran on the legacy stream; finish them before the stage stream runs
  CU(cudaDeviceSynchronize());
  return LC_OK;
}

// ---- training-mode building blocks ------------------------------------------------------------

GemmProblem bf16_problem(uint64_t m, uint64_t n, uint64_t k) {
  GemmProblem g;
  g.m = m;
  g.n = n;
  g.k = k;
  g.batch = 1;
  g.in_dtype = LC_BF16;
  g.c_dtype = LC_BF16;
  g.reserve_sms = 4;  // room for the NCCL transfer kernels next to the persistent GEMM
  return g;
}

// H[l+1][rows] = relu(H[l][rows] @ Wb_l)
GemmProblem fwd_problem(lc_pipeline* p, uint64_t l, uint64_t row0, uint64_t rows) {
  const uint64_t k = p->win(l), n = p->wout(l);
  GemmProblem g = bf16_problem(rows, n, k);
  g.a.data = p->H[l];
  g.a.offset = row0 * k;
  g.a.mn = rows;
  g.a.k = k;
  g.a.mn_stride = (int64_t)k;
  g.a.k_stride = 1;
  g.b.data = p->wb[l];  // [k][n] row-major: element (n, k) at k*n_cols + n
  g.b.mn = n;
  g.b.k = k;
  g.b.mn_stride = 1;
  g.b.k_stride = (int64_t)n;
  g.c = p->H[l + 1];
  g.c_offset = row0 * n;
  g.c_m_stride = (int64_t)n;
  g.c_n_stride = 1;
  g.relu = 1;
  return g;
}

// out[rows] = (dP[l][rows] @ Wb_l^T) where H[l][rows] > 0
GemmProblem dgrad_problem(lc_pipeline* p, uint64_t l, uint64_t row0, uint64_t rows, void* out) {
  const uint64_t k = p->wout(l), n = p->win(l);
  GemmProblem g = bf16_problem(rows, n, k);
  g.a.data = p->dP[l];
  g.a.offset = row0 * k;
  g.a.mn = rows;
  g.a.k = k;
  g.a.mn_stride = (int64_t)k;
  g.a.k_stride = 1;
  g.b.data = p->wb[l];  // B[k=j][n=i] = W[i][j]: element (n=i, k=j) at i*k + j
  g.b.mn = n;
  g.b.k = k;
  g.b.mn_stride = (int64_t)k;
  g.b.k_stride = 1;
  g.c = out;
  g.c_offset = row0 * n;
  g.c_m_stride = (int64_t)n;
  g.c_n_stride = 1;
  g.epi = 1;
  g.aux = p->H[l];  // the layer's input, same [B, n] layout as the output
  return g;
}

// The stage's layer loop of one microbatch as one chain launch when the products allow it
// (the weights are read-only between the steps' weight updates), else one launch per layer.
lc_status run_products(lc_pipeline* p, cudaStream_t s, const std::vector<GemmProblem>& probs) {
  if (probs.empty()) return LC_OK;
  bool chained = false;
  // with K compute streams, K chains share the GPU: each takes 1/K of the SMs' CTA pairs
  // (16 of 64 at width 8192 and K = 4, four tiles per pair)
  const int cap = p->n_streams > 1 ? (int)std::max<int64_t>(1, (p->ctx->sm_count - 4) / (2 * p->n_streams)) : 0;
  lc_status st = gemm_chain_run(p->ctx, s, probs.data(), (int)probs.size(), true, cap, &chained);
  if (st || chained) return st;
  for (const GemmProblem& g : probs)
    if ((st = gemm_run(p->ctx, s, g, nullptr, false))) return st;
  return LC_OK;
}

// Microbatches per product (training mode).  The forwards only read weights nobody writes before
// the step's weight updates, and B(m) needs nothing but F(m) (and, on a later stage, the
// gradient of m from the next stage), so consecutive microbatches run as one taller product per
// layer without changing any result: each group product keeps the one-microbatch product's split
// count and orientation, so every element sees the same operations in the same order.  The
// schedule is then 1F1B over the groups (local_order over microbatches / fuse units), each group
// crossing a stage boundary as one transfer of its rows.  LC_PIPE_FUSE=1 turns it off.
lc_status decide_fuse(lc_pipeline* p) {
  static const int env_fuse = [] {
    const char* e = getenv("LC_PIPE_FUSE");  // microbatches per product on one stage (1, 2 or 4)
    return e ? atoi(e) : 0;
  }();
  static const bool env_narrow = [] {
    const char* e = getenv("LC_PIPE_GROUP_TILE");  // "0": keep the one-microbatch tile width
    return e != nullptr && e[0] == '0';
  }();
  const uint64_t mbs = p->cfg.microbatches, mb = p->cfg.microbatch;
  uint64_t want = env_fuse == 1 || env_fuse == 2 || env_fuse == 4 ? (uint64_t)env_fuse : kFuseDefault;
  while (want > 1 && mbs % want != 0) want /= 2;
  if (!p->train_mode) want = 1;
  if (want > 1) {
    // Each group product keeps the one-microbatch product's split count and orientation, so
    // every element is computed by the same operations in the same order.
    p->fwd_shape.assign(p->count, {});
    p->dgrad_shape.assign(p->count, {});
    for (uint64_t l = 0; l < p->count; l++) {
      lc_pipeline::Shape& f = p->fwd_shape[l];
      lc_status st = gemm_plan_shape(p->ctx, fwd_problem(p, l, 0, mb), &f.bn, &f.splits, &f.swap);
      if (st) return st;
      if (l > 0 || !p->is_first()) {
        lc_pipeline::Shape& d = p->dgrad_shape[l];
        st = gemm_plan_shape(p->ctx, dgrad_problem(p, l, 0, mb, l > 0 ? p->dP[l - 1] : p->gsend), &d.bn, &d.splits,
                             &d.swap);
        if (st) return st;
      }
      // A wider tile covers the group's rows (up to 256), so each weight tile is read by one CTA
      // pair for the whole group; with 64-wide tiles each CTA also re-reads its slice of the
      // activations, which made the per-SM load, not the DRAM, the limit.
      if (!env_narrow)
        for (lc_pipeline::Shape* sh : {&p->fwd_shape[l], &p->dgrad_shape[l]})
          if (sh->bn == 64 && sh->swap > 0) sh->bn = (int32_t)std::min<uint64_t>(256, 64 * want);
    }
  }
  p->fuse = want;
  return LC_OK;
}

// `g` over a group of microbatches, planned from the one-microbatch product's shape
GemmProblem shaped(GemmProblem g, const lc_pipeline::Shape& sh) {
  g.bn_hint = sh.bn;
  g.splits_hint = sh.splits;
  g.swap_hint = sh.swap;
  return g;
}

// W_l -= lr * H[l]^T @ dP[l] (K = B), Wb_l = bf16(W_l); or dW_l = H[l]^T @ dP[l] when lr == 0
lc_status wgrad_layer(lc_pipeline* p, uint64_t l) {
  const uint64_t m = p->win(l), n = p->wout(l), k = p->B;
  GemmProblem g = bf16_problem(m, n, k);
  g.a.data = p->H[l];  // A[m=i][k=b] = H[b][i]
  g.a.mn = m;
  g.a.k = k;
  g.a.mn_stride = 1;
  g.a.k_stride = (int64_t)m;
  g.b.data = p->dP[l];  // B[k=b][n=j] = dP[b][j]
  g.b.mn = n;
  g.b.k = k;
  g.b.mn_stride = 1;
  g.b.k_stride = (int64_t)n;
  g.c_m_stride = (int64_t)n;
  g.c_n_stride = 1;
  if (p->cfg.lr != 0.0f) {
    g.epi = 2;
    g.aux = p->master[l];
    g.aux2 = p->wb[l];
    g.lr = p->cfg.lr;
    g.c = p->master[l];  // unused by the SGD epilogue; keeps the pointer valid
    g.c_dtype = LC_F32;
  } else {
    g.c = p->dw[l];
    g.c_dtype = LC_F32;
  }
  return gemm_run(p->ctx, p->comp(), g, nullptr, false);
}

// ---- reference-mode building blocks (the reference's Backend call sequence) -------------------

// pre = x @ W, act = gelu(pre) (crates/pipeline/src/lib.rs:176-178).  GELU layers do both in one
// product (the fused GELU epilogue stores pre and act, the same bits as gemm then gelu); ReLU
// layers run the gemm and the standalone relu.
lc_status ref_forward(lc_pipeline* p, uint64_t l, uint64_t row0, uint64_t rows) {
  const uint64_t k = p->win(l), n = p->wout(l);
  lc_view x = matrix_view((float*)p->H[l] + row0 * k, LC_F32, rows, k, rows * k * 4);
  lc_view w = matrix_view(p->master[l], LC_F32, k, n, k * n * 4);
  lc_view pre = matrix_view(p->pre[l] + row0 * n, LC_F32, rows, n, rows * n * 4);
  lc_view act = matrix_view((float*)p->H[l + 1] + row0 * n, LC_F32, rows, n, rows * n * 4);
  if (p->cfg.activation == 0) {
    lc_epilogue e{};
    e.kind = LC_EPI_GELU;
    e.aux2 = &pre;
    return lc_encode_gemm_fused(p->ctx, p->comp(), 1.0f, &x, &w, 0.0f, &act, &e);
  }
  lc_status st = lc_backend_gemm(p->ctx, p->comp(), &x, &w, &pre, 1.0f, 0.0f);
  if (st) return st;
  return lc_relu(p->ctx, p->comp(), &pre, &act);
}

// The stage's backward of one microbatch in the reference's order (crates/pipeline/src/lib.rs:
// 204-227): for l = count-1 .. 0, dpre = act'(pre[l]) * g, dW[l] += x^T dpre (beta = 1), g = dpre @
// W^T for the layer below (sent to the previous stage after layer 0).  `g` is the gradient at the
// stage's output (f32 [rows, n]).  GELU layers fold each act' into the product that makes its g
// (the fused GELU-backward epilogue: the same bits as the product followed by gelu_backward), so
// only the top layer's act' runs as its own kernel; dpre alternates between two scratch buffers.
lc_status ref_backward_stage(lc_pipeline* p, uint64_t row0, uint64_t rows, const float* g) {
  const bool gelu = p->cfg.activation == 0;
  float* bufs[2] = {(float*)p->dbuf, (float*)p->dbuf2};
  int cur = 0;
  lc_status st = LC_OK;
  {
    const uint64_t l = p->count - 1, n = p->wout(l);
    lc_view pre = matrix_view(p->pre[l] + row0 * n, LC_F32, rows, n, rows * n * 4);
    lc_view gv = matrix_view(const_cast<float*>(g), LC_F32, rows, n, rows * n * 4);
    lc_view dpre = matrix_view(bufs[cur], LC_F32, rows, n, rows * n * 4);
    st = gelu ? lc_gelu_backward(p->ctx, p->comp(), &pre, &gv, &dpre) : lc_relu_backward(p->ctx, p->comp(), &pre, &gv, &dpre);
    if (st) return st;
  }
  for (uint64_t l = p->count; l-- > 0;) {
    const uint64_t k = p->win(l), n = p->wout(l);
    lc_view dpre = matrix_view(bufs[cur], LC_F32, rows, n, rows * n * 4);
    // dW[k, n] += x^T [k, rows] @ dpre [rows, n]  (:218, beta = 1)
    lc_view xt{};
    xt.data = (float*)p->H[l] + row0 * k;
    xt.buffer_bytes = rows * k * 4;
    xt.dtype = LC_F32;
    xt.rank = 2;
    xt.shape[0] = k;
    xt.shape[1] = rows;
    xt.strides[0] = 1;
    xt.strides[1] = k;
    lc_view dwv = matrix_view(p->dw[l], LC_F32, k, n, k * n * 4);
    if ((st = lc_backend_gemm(p->ctx, p->comp(), &xt, &dpre, &dwv, 1.0f, 1.0f))) return st;
    if (l == 0 && p->is_first()) break;  // the reference computes and discards this dx
    // dX[rows, k] = dpre [rows, n] @ W^T [n, k]  (:220)
    lc_view wt{};
    wt.data = p->master[l];
    wt.buffer_bytes = k * n * 4;
    wt.dtype = LC_F32;
    wt.rank = 2;
    wt.shape[0] = n;
    wt.shape[1] = k;
    wt.strides[0] = 1;
    wt.strides[1] = n;
    if (l == 0) {
      lc_view dx = matrix_view((float*)p->gsend + row0 * k, LC_F32, rows, k, rows * k * 4);
      return lc_backend_gemm(p->ctx, p->comp(), &dpre, &wt, &dx, 1.0f, 0.0f);
    }
    // the layer below's dpre from this layer's dx
    lc_view below_pre = matrix_view(p->pre[l - 1] + row0 * k, LC_F32, rows, k, rows * k * 4);
    lc_view other = matrix_view(bufs[cur ^ 1], LC_F32, rows, k, rows * k * 4);
    if (gelu) {
      lc_epilogue e{};
      e.kind = LC_EPI_GELU_BACKWARD;
      e.aux = &below_pre;
      st = lc_encode_gemm_fused(p->ctx, p->comp(), 1.0f, &dpre, &wt, 0.0f, &other, &e);
      cur ^= 1;
    } else {
      // dx into the other buffer, then the layer below's dpre over this one (its last readers,
      // the two products above, precede it on the stream)
      st = lc_backend_gemm(p->ctx, p->comp(), &dpre, &wt, &other, 1.0f, 0.0f);
      lc_view below = matrix_view(bufs[cur], LC_F32, rows, k, rows * k * 4);
      if (!st) st = lc_relu_backward(p->ctx, p->comp(), &below_pre, &other, &below);
    }
    if (st) return st;
  }
  return LC_OK;
}

lc_status wait_step(lc_pipeline* p) {
  using clock = std::chrono::steady_clock;
  const auto t0 = clock::now();
  const int64_t limit_ms = p->cfg.timeout_ms > 0 ? p->cfg.timeout_ms : 60000;
  for (;;) {
    cudaError_t q = cudaEventQuery(p->ev_end);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return cuda_fail(q, "pipeline step");
    for (ncclComm_t c : {p->comm_fwd, p->comm_bwd}) {
      if (c == nullptr) continue;
      ncclResult_t ar = ncclSuccess;
      if (nccl().CommGetAsyncError(c, &ar) == ncclSuccess && ar != ncclSuccess && ar != ncclInProgress) {
        nccl().CommAbort(p->comm_fwd);
        nccl().CommAbort(p->comm_bwd);
        p->comm_fwd = p->comm_bwd = nullptr;
        p->aborted = true;
        return nccl_fail(ar, "peer transfer failed");
      }
    }
    if (std::chrono::duration_cast<std::chrono::milliseconds>(clock::now() - t0).count() > limit_ms) {
      if (p->comm_fwd) nccl().CommAbort(p->comm_fwd);
      if (p->comm_bwd) nccl().CommAbort(p->comm_bwd);
      p->comm_fwd = p->comm_bwd = nullptr;
      p->aborted = true;
      return fail(LC_ERR_TRANSPORT, "pipeline step did not finish within timeout_ms; a peer is gone");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  CU(cudaEventElapsedTime(&p->last_ms, p->ev_start, p->ev_end));
  return lc_sync(p->ctx, nullptr);
}

}  // namespace

extern "C" {

lc_status lc_pipeline_unique_id(uint8_t id[LC_PIPELINE_ID_BYTES]) {
  static_assert(sizeof(ncclUniqueId) == LC_PIPELINE_ID_BYTES, "NCCL unique id size");
  if (!nccl().ok) return fail(LC_ERR_TRANSPORT, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  NC(nccl().GetUniqueId(&u));
  memcpy(id, &u, sizeof(u));
  return LC_OK;
}

lc_status lc_pipeline_create(const lc_pipeline_config* cfg, const uint8_t id[LC_PIPELINE_ID_BYTES], int32_t rank,
                             int32_t world, int32_t device, lc_pipeline** out) {
  if (cfg == nullptr || out == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (world < 1 || rank < 0 || rank >= world) return fail(LC_ERR_SCHEDULE, "rank outside the world");
  if (cfg->microbatches == 0 || cfg->microbatch == 0) return fail(LC_ERR_SCHEDULE, "no microbatches");
  const bool train = cfg->compute_dtype == LC_BF16;
  if (!train && cfg->compute_dtype != LC_F32) return fail(LC_ERR_DTYPE, "compute dtype is f32 or bf16");
  if (train && (cfg->activation != 1 || cfg->loss != 1))
    return fail(LC_ERR_INVALID_ARGUMENT, "training mode is ReLU layers with the MSE loss");
  if (!train && (cfg->loss != 0 || cfg->lr != 0.0f))
    return fail(LC_ERR_INVALID_ARGUMENT, "reference mode takes dy from the caller and applies no optimizer");
  std::vector<uint64_t> owners(cfg->layers);
  lc_status st = lc_contiguous_placement(cfg->layers, (uint64_t)world, owners.data());
  if (st) return st;
  auto* p = new lc_pipeline();
  p->cfg = *cfg;
  p->rank = rank;
  p->world = world;
  p->device = device;
  p->train_mode = train;
  for (uint64_t l = 0; l <= cfg->layers; l++) p->widths.push_back(cfg->widths ? cfg->widths[l] : cfg->width);
  p->cfg.widths = nullptr;
  for (uint64_t l = 0; l < cfg->layers; l++)
    if (owners[l] == (uint64_t)rank) {
      if (p->count == 0) p->first = l;
      p->count++;
    }
  if (train)
    for (uint64_t w : p->widths)
      if (w % 8 != 0) {
        delete p;
        return fail(LC_ERR_SHAPE, "training mode widths must be multiples of 8 (16-byte rows)");
      }
  if ((st = lc_context_create(device, &p->ctx))) {
    delete p;
    return st;
  }
  if ((st = setup(p))) {
    lc_pipeline_destroy(p);
    return st;
  }
  if (world > 1) {
    if (id == nullptr) {
      lc_pipeline_destroy(p);
      return fail(LC_ERR_INVALID_ARGUMENT, "null communicator id");
    }
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    if (!nccl().ok) {
      lc_pipeline_destroy(p);
      return fail(LC_ERR_TRANSPORT, "libnccl.so.2 could not be loaded");
    }
    // NCCL's transfer kernels share the GPU with the layer chains (cooperative launches sized to
    // leave 4 SMs free).  Capping them at two CTAs each, so that a spinning receive could never
    // hold SMs a chain needs, measured no better on 2 B200s (59.6k samples/s either way) and
    // slower on 4 (97.3k against 104.6k): NCCL keeps its own count unless LC_PIPE_NCCL_CTAS asks.
    static const int env_ctas = [] {
      const char* e = getenv("LC_PIPE_NCCL_CTAS");  // tuning override: CTAs per NCCL kernel, 0 = NCCL's choice
      return e ? atoi(e) : -1;
    }();
    const int ctas = env_ctas >= 0 ? env_ctas : kNcclCtas;
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    if (ctas > 0) {
      cfg.minCTAs = 1;
      cfg.maxCTAs = ctas;
    }
    ncclResult_t r = nccl().CommInitRankConfig(&p->comm_fwd, world, u, rank, &cfg);
    if (r == ncclSuccess) r = nccl().CommSplit(p->comm_fwd, 0, rank, &p->comm_bwd, &cfg);
    if (r != ncclSuccess) {
      lc_pipeline_destroy(p);
      return nccl_fail(r, "communicator setup");
    }
  }
  *out = p;
  return LC_OK;
}

lc_status lc_pipeline_destroy(lc_pipeline* p) {
  if (p == nullptr) return LC_OK;
  if (p->ctx) {
    cudaSetDevice(p->device);
    cudaDeviceSynchronize();
  }
  if (p->comm_bwd) nccl().CommDestroy(p->comm_bwd);
  if (p->comm_fwd) nccl().CommDestroy(p->comm_fwd);
  for (auto* v : {&p->master, &p->dw, &p->pre})
    for (float* q : *v) cudaFree(q);
  for (auto* v : {&p->wb, &p->H, &p->dP})
    for (void* q : *v) cudaFree(q);
  for (void* q : {p->gsend, p->dbuf, p->dbuf2, (void*)p->x_dev, (void*)p->t_dev, (void*)p->part, (void*)p->loss_dev})
    if (q) cudaFree(q);
  if (p->loss_host) cudaFreeHost(p->loss_host);
  for (auto* v : {&p->ev_fr, &p->ev_fd, &p->ev_br, &p->ev_bd, &p->ev_fdone})
    for (auto e : *v) cudaEventDestroy(e);
  for (auto e : {p->ev_start, p->ev_end, p->ev_fwd_join, p->ev_bwd_join, p->ev_inputs})
    if (e) cudaEventDestroy(e);
  for (auto e : p->ev_work_join) cudaEventDestroy(e);
  for (auto* v : {&p->ev_t0, &p->ev_t1})
    for (auto e : *v) cudaEventDestroy(e);
  for (auto q : p->s_work)
    if (q) cudaStreamDestroy(q);
  if (p->s_fwd) cudaStreamDestroy(p->s_fwd);
  if (p->s_bwd) cudaStreamDestroy(p->s_bwd);
  if (p->ctx) lc_context_destroy(p->ctx);
  delete p;
  return LC_OK;
}

lc_status lc_pipeline_local_layers(lc_pipeline* p, uint64_t* first, uint64_t* count) {
  if (!p || !first || !count) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  *first = p->first;
  *count = p->count;
  return LC_OK;
}

lc_status lc_pipeline_set_weight(lc_pipeline* p, uint64_t index, const float* host_w) {
  if (!p || !host_w || index >= p->count) return fail(LC_ERR_INVALID_ARGUMENT, "bad layer index");
  cudaSetDevice(p->device);
  const uint64_t n = p->win(index) * p->wout(index);
  lc_status st = copy_sync(p, p->master[index], host_w, n * 4, cudaMemcpyHostToDevice);
  if (st) return st;
  if (p->train_mode) {
    to_bf16_kernel<<<blocks_for(p->ctx, n), 256, 0, p->comp()>>>(p->master[index], (uint16_t*)p->wb[index], n);
    record_launch(p->ctx, "pipeline_to_bf16");
    CU(cudaStreamSynchronize(p->comp()));
  }
  return LC_OK;
}

lc_status lc_pipeline_init_weights(lc_pipeline* p, uint64_t seed, float stddev) {
  if (!p) return fail(LC_ERR_INVALID_ARGUMENT, "null pipeline");
  cudaSetDevice(p->device);
  for (uint64_t l = 0; l < p->count; l++) {
    const uint64_t n = p->win(l) * p->wout(l);
    normal_init_kernel<<<blocks_for(p->ctx, n), 256, 0, p->comp()>>>(
        p->master[l], p->train_mode ? (uint16_t*)p->wb[l] : nullptr, n, seed + p->first + l, stddev);
    record_launch(p->ctx, "pipeline_init_weights");
  }
  CU(cudaStreamSynchronize(p->comp()));
  return LC_OK;
}

lc_status lc_pipeline_get_weight(lc_pipeline* p, uint64_t index, float* host_w) {
  if (!p || !host_w || index >= p->count) return fail(LC_ERR_INVALID_ARGUMENT, "bad layer index");
  cudaSetDevice(p->device);
  return copy_sync(p, host_w, p->master[index], p->win(index) * p->wout(index) * 4, cudaMemcpyDeviceToHost);
}

lc_status lc_pipeline_get_grad(lc_pipeline* p, uint64_t index, float* host_dw) {
  if (!p || !host_dw || index >= p->count) return fail(LC_ERR_INVALID_ARGUMENT, "bad layer index");
  if (p->dw.empty())
    return fail(LC_ERR_INVALID_ARGUMENT, "the gradient is fused into the SGD update (lr != 0); nothing to read");
  cudaSetDevice(p->device);
  return copy_sync(p, host_dw, p->dw[index], p->win(index) * p->wout(index) * 4, cudaMemcpyDeviceToHost);
}

lc_status lc_pipeline_get_output(lc_pipeline* p, float* host_y) {
  if (!p || !host_y) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (!p->is_last()) return fail(LC_ERR_SCHEDULE, "only the last stage holds the output");
  cudaSetDevice(p->device);
  const uint64_t n = p->B * p->widths.back();
  if (!p->train_mode) return copy_sync(p, host_y, p->H[p->count], n * 4, cudaMemcpyDeviceToHost);
  std::vector<uint16_t> h(n);
  lc_status st = copy_sync(p, h.data(), p->H[p->count], n * 2, cudaMemcpyDeviceToHost);
  if (st) return st;
  for (uint64_t i = 0; i < n; i++) {
    uint32_t b = ((uint32_t)h[i]) << 16;
    memcpy(&host_y[i], &b, 4);
  }
  return LC_OK;
}

lc_status lc_pipeline_set_trace(lc_pipeline* p, int32_t on) {
  if (!p) return fail(LC_ERR_INVALID_ARGUMENT, "null pipeline");
  cudaSetDevice(p->device);
  if (on && p->ev_t0.empty()) {
    const size_t n = 2 * p->cfg.microbatches + p->count;
    p->ev_t0.resize(n);
    p->ev_t1.resize(n);
    for (auto* v : {&p->ev_t0, &p->ev_t1})
      for (auto& e : *v) CU(cudaEventCreate(&e));
  }
  p->trace = on != 0;
  p->trace_rec.clear();
  return LC_OK;
}

lc_status lc_pipeline_trace(lc_pipeline* p, float* out, uint64_t cap, uint64_t* n) {
  if (!p || !n) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  const uint64_t have = p->trace_rec.size() / 4;
  *n = have;
  if (out == nullptr) return LC_OK;
  if (cap < have) return fail(LC_ERR_INVALID_ARGUMENT, "trace buffer holds fewer records than the step made");
  memcpy(out, p->trace_rec.data(), p->trace_rec.size() * sizeof(float));
  return LC_OK;
}

lc_status lc_pipeline_last_step_ms(lc_pipeline* p, float* ms) {
  if (!p || !ms) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  *ms = p->last_ms;
  return LC_OK;
}

void* lc_pipeline_stream(lc_pipeline* p) { return p ? p->comp() : nullptr; }

uint64_t lc_pipeline_debug_launches(lc_pipeline* p) { return p ? lc_debug_launches(p->ctx) : 0; }

lc_status lc_pipeline_step(lc_pipeline* p, const float* x, const float* target_or_dy, int32_t inputs_on_device,
                           float* loss) {
  if (!p) return fail(LC_ERR_INVALID_ARGUMENT, "null pipeline");
  if (p->aborted) return fail(LC_ERR_TRANSPORT, "the pipeline's communicators were aborted");
  if (p->is_first() && x == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "rank 0 needs the inputs");
  if (p->is_last() && target_or_dy == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "the last rank needs targets or dy");
  cudaSetDevice(p->device);
  const uint64_t mbs = p->cfg.microbatches, mb = p->cfg.microbatch;
  if (p->fuse == 0) {
    const lc_status fs = decide_fuse(p);
    if (fs) return fs;
  }
  const uint64_t fuse = p->fuse;
  std::vector<int64_t> order(2 * mbs);
  uint64_t n_ops = 0;
  // 1F1B over groups of `fuse` microbatches: op +-(u + 1) of the group schedule covers
  // microbatches u * fuse .. u * fuse + fuse - 1, stored here as +-(first microbatch + 1)
  lc_status st = lc_local_order((uint64_t)p->world, (uint64_t)p->rank, mbs / fuse, order.data(), order.size(), &n_ops);
  if (st) return st;
  for (uint64_t i = 0; i < n_ops; i++) {
    const int64_t u = (order[i] > 0 ? order[i] : -order[i]) - 1;
    order[i] = (order[i] > 0 ? 1 : -1) * (u * (int64_t)fuse + 1);
  }
  cudaStream_t cs = p->comp();
  const ncclDataType_t nt = p->train_mode ? ncclBfloat16 : ncclFloat32;
  const uint64_t w0 = p->win(0), wl = p->wout(p->count - 1);
  const size_t es = p->es();
  CU(cudaEventRecord(p->ev_start, cs));
  // fork the transfer streams from the step start
  CU(cudaStreamWaitEvent(p->s_fwd, p->ev_start, 0));
  CU(cudaStreamWaitEvent(p->s_bwd, p->ev_start, 0));
  const cudaMemcpyKind kind = inputs_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (p->is_first()) CU(cudaMemcpyAsync(p->x_dev, x, p->B * p->widths[0] * 4, kind, cs));
  if (p->is_last()) CU(cudaMemcpyAsync(p->t_dev, target_or_dy, p->B * p->widths.back() * 4, kind, cs));
  CU(cudaEventRecord(p->ev_inputs, cs));
  for (cudaStream_t q : p->s_work) CU(cudaStreamWaitEvent(q, p->ev_inputs, 0));
  const float n_total = (float)(p->B * p->widths.back());

  for (uint64_t i = 0; i < n_ops && !st; i++) {
    const bool fwd = order[i] > 0;
    const uint64_t m = (uint64_t)(fwd ? order[i] : -order[i]) - 1;
    const uint64_t row0 = m * mb;
    const uint64_t rows = fuse * mb;  // this op's microbatches m .. m+fuse-1 are adjacent rows
    if (fwd) {
      const cudaStream_t fs = p->fwd_stream(m / fuse);
      void* in = (uint8_t*)p->H[0] + row0 * w0 * es;
      if (p->is_first()) {
        if (p->train_mode) {
          to_bf16_kernel<<<blocks_for(p->ctx, rows * w0), 256, 0, fs>>>(p->x_dev + row0 * w0, (uint16_t*)in, rows * w0);
          record_launch(p->ctx, "pipeline_input_to_bf16");
        } else {
          CU(cudaMemcpyAsync(in, p->x_dev + row0 * w0, rows * w0 * 4, cudaMemcpyDeviceToDevice, fs));
        }
      } else {
        NC(nccl().Recv(in, rows * w0, nt, p->rank - 1, p->comm_fwd, p->s_fwd));
        CU(cudaEventRecord(p->ev_fr[m], p->s_fwd));
        CU(cudaStreamWaitEvent(fs, p->ev_fr[m], 0));
      }
      const uint64_t ti = i;  // trace slot of this op
      if (p->trace) CU(cudaEventRecord(p->ev_t0[ti], fs));
      if (p->train_mode) {
        std::vector<GemmProblem> probs;
        for (uint64_t l = 0; l < p->count; l++)
          probs.push_back(fuse > 1 ? shaped(fwd_problem(p, l, row0, rows), p->fwd_shape[l]) : fwd_problem(p, l, row0, mb));
        st = run_products(p, fs, probs);
      } else {
        for (uint64_t j = 0; j < fuse && !st; j++)
          for (uint64_t l = 0; l < p->count && !st; l++) st = ref_forward(p, l, row0 + j * mb, mb);
      }
      if (st) break;
      void* outp = (uint8_t*)p->H[p->count] + row0 * wl * es;
      if (!p->is_last()) {
        CU(cudaEventRecord(p->ev_fd[m], fs));
        CU(cudaStreamWaitEvent(p->s_fwd, p->ev_fd[m], 0));
        NC(nccl().Send(outp, rows * wl, nt, p->rank + 1, p->comm_fwd, p->s_fwd));
      } else if (p->train_mode) {
        // one launch per microbatch: its loss partials are summed exactly as without grouping
        for (uint64_t j = 0; j < fuse; j++) {
          const uint64_t r = row0 + j * mb;
          mse_relu_kernel<<<kMseBlocks, kMseThreads, 0, fs>>>((const uint16_t*)p->H[p->count] + r * wl, p->t_dev + r * wl,
                                                            (uint16_t*)p->dP[p->count - 1] + r * wl, mb * wl, n_total,
                                                            p->part + (m + j) * kMseBlocks);
          record_launch(p->ctx, "pipeline_mse_relu");
        }
      }
      CU(cudaEventRecord(p->ev_fdone[m], fs));
      if (p->trace) CU(cudaEventRecord(p->ev_t1[ti], fs));
    } else {
      // backward of microbatch m on its own stream, after its forward (activations, masks, the
      // loss gradient) is complete
      const cudaStream_t bs = p->back_stream(m / fuse);
      CU(cudaStreamWaitEvent(bs, p->ev_fdone[m], 0));
      // incoming gradient for the stage's last layer
      const float* g_ref = nullptr;
      if (!p->is_last()) {
        void* gin = (uint8_t*)p->dP[p->train_mode ? p->count - 1 : 0] + row0 * wl * es;
        NC(nccl().Recv(gin, rows * wl, nt, p->rank + 1, p->comm_bwd, p->s_bwd));
        CU(cudaEventRecord(p->ev_br[m], p->s_bwd));
        CU(cudaStreamWaitEvent(bs, p->ev_br[m], 0));
        g_ref = (const float*)gin;
      } else {
        g_ref = p->t_dev + row0 * wl;  // reference mode: dy
      }
      if (p->trace) CU(cudaEventRecord(p->ev_t0[i], bs));
      if (p->train_mode) {
        std::vector<GemmProblem> probs;
        for (uint64_t l = p->count; l-- > 0;) {
          if (l == 0 && p->is_first()) continue;  // rank 0 discards layer 0's input gradient
          GemmProblem g = dgrad_problem(p, l, row0, rows, l > 0 ? p->dP[l - 1] : p->gsend);
          probs.push_back(fuse > 1 ? shaped(g, p->dgrad_shape[l]) : g);
        }
        st = run_products(p, bs, probs);
      } else {
        st = ref_backward_stage(p, row0, mb, g_ref);
      }
      if (st) break;
      if (p->trace) CU(cudaEventRecord(p->ev_t1[i], bs));
      if (!p->is_first()) {
        CU(cudaEventRecord(p->ev_bd[m], bs));
        CU(cudaStreamWaitEvent(p->s_bwd, p->ev_bd[m], 0));
        NC(nccl().Send((uint8_t*)p->gsend + row0 * w0 * es, rows * w0, nt, p->rank - 1, p->comm_bwd, p->s_bwd));
      }
    }
  }
  // the weight updates read every microbatch's gradients: join the compute streams first
  for (size_t i = 0; i < p->s_work.size(); i++) {
    CU(cudaEventRecord(p->ev_work_join[i], p->s_work[i]));
    CU(cudaStreamWaitEvent(cs, p->ev_work_join[i], 0));
  }
  if (!st && p->train_mode)
    for (uint64_t l = 0; l < p->count && !st; l++) {
      if (p->trace) CU(cudaEventRecord(p->ev_t0[n_ops + l], cs));
      st = wgrad_layer(p, l);
      if (p->trace) CU(cudaEventRecord(p->ev_t1[n_ops + l], cs));
    }
  if (!st && p->train_mode && p->is_last()) {
    loss_reduce_kernel<<<1, kMseThreads, 0, cs>>>(p->part, (int)(kMseBlocks * mbs), n_total, p->loss_dev);
    record_launch(p->ctx, "pipeline_loss_reduce");
    CU(cudaMemcpyAsync(p->loss_host, p->loss_dev, sizeof(float), cudaMemcpyDeviceToHost, cs));
  }
  // join the transfer streams before the step-end event
  CU(cudaEventRecord(p->ev_fwd_join, p->s_fwd));
  CU(cudaEventRecord(p->ev_bwd_join, p->s_bwd));
  CU(cudaStreamWaitEvent(cs, p->ev_fwd_join, 0));
  CU(cudaStreamWaitEvent(cs, p->ev_bwd_join, 0));
  CU(cudaEventRecord(p->ev_end, cs));
  lc_status wst = wait_step(p);
  if (st) return st;
  if (wst) return wst;
  if (p->trace) {
    p->trace_rec.clear();
    const uint64_t n_w = p->train_mode ? p->count : 0;
    for (uint64_t i = 0; i < n_ops + n_w; i++) {
      float t0 = 0.0f, t1 = 0.0f;
      CU(cudaEventElapsedTime(&t0, p->ev_start, p->ev_t0[i]));
      CU(cudaEventElapsedTime(&t1, p->ev_start, p->ev_t1[i]));
      const bool op = i < n_ops;
      p->trace_rec.insert(p->trace_rec.end(),
                          {op ? (order[i] > 0 ? 1.0f : -1.0f) : 2.0f,
                           op ? (float)((order[i] > 0 ? order[i] : -order[i]) - 1) : (float)(p->first + i - n_ops), t0,
                           t1});
    }
  }
  if (loss) *loss = (p->train_mode && p->is_last()) ? *p->loss_host : 0.0f;
  return LC_OK;
}

}  // extern "C"
