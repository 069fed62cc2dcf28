// core.cpp -- context, errors, launch log, scratch, and strided-view metadata.
//
// The view rules restate the reference's data model (src/abi.rs) and the per-op checks that
// every primitive shares (overlap, injective destination, contiguity).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "internal.h"

namespace {
thread_local std::string g_last_error;
constexpr size_t kLaunchRing = 4096;
}  // namespace

namespace lc {

lc_status fail(lc_status code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

lc_status cuda_fail(cudaError_t e, const char* what) {
  return fail(LC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

void record_launch(lc_context* ctx, const char* name) {
  uint64_t i = ctx->launches.fetch_add(1);
  std::lock_guard<std::mutex> g(ctx->names_mu);
  if (ctx->names.size() < kLaunchRing) ctx->names.resize(kLaunchRing, nullptr);
  ctx->names[i % kLaunchRing] = name;
}

lc_status scratch_alloc(lc_context* ctx, cudaStream_t s, size_t bytes, void** out) {
  (void)ctx;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMallocAsync(out, bytes, s);
  if (e != cudaSuccess) return cuda_fail(e, "scratch cudaMallocAsync");
  return LC_OK;
}

void scratch_free(void* p, cudaStream_t s) {
  if (p != nullptr) cudaFreeAsync(p, s);
}

size_t dtype_size(int32_t dtype) {
  switch (dtype) {
    case LC_F32:
    case LC_U32:
    case LC_I32:
      return 4;
    case LC_F16:
    case LC_BF16:
    case LC_U16:
      return 2;
    case LC_C32:
    case LC_F64:
      return 8;
    case LC_C64:
      return 16;
    default:
      return 0;
  }
}

bool dtype_known(int32_t dtype) { return dtype_size(dtype) != 0; }

uint64_t numel(const lc_view& v) {
  uint64_t n = 1;
  for (int d = 0; d < v.rank; d++) n *= v.shape[d];
  return n;
}

bool is_empty(const lc_view& v) {
  for (int d = 0; d < v.rank; d++)
    if (v.shape[d] == 0) return true;
  return false;
}

bool max_index(const lc_view& v, uint64_t* last) {
  uint64_t acc = v.offset;
  for (int d = 0; d < v.rank; d++) {
    if (v.shape[d] == 0) return false;
    uint64_t step;
    if (__builtin_mul_overflow(v.shape[d] - 1, v.strides[d], &step)) return false;
    if (__builtin_add_overflow(acc, step, &acc)) return false;
  }
  *last = acc;
  return true;
}

lc_status validate(const lc_view& v, const char* name) {
  if (!dtype_known(v.dtype)) return fail(LC_ERR_INVALID_ARGUMENT, std::string(name) + ": unknown element type");
  if (v.rank < 0 || v.rank > LC_MAX_RANK)
    return fail(LC_ERR_INVALID_ARGUMENT, std::string(name) + ": rank " + std::to_string(v.rank) + " outside 0..8");
  size_t es = dtype_size(v.dtype);
  if (v.data == nullptr && v.buffer_bytes != 0)
    return fail(LC_ERR_INVALID_ARGUMENT, std::string(name) + ": null buffer");
  if (reinterpret_cast<uintptr_t>(v.data) % std::min<size_t>(es, 16) != 0)
    return fail(LC_ERR_INVALID_ARGUMENT, std::string(name) + ": buffer base is misaligned for the element type");
  uint64_t capacity = v.buffer_bytes / es;
  if (is_empty(v)) {
    if (v.offset <= capacity) return LC_OK;
    return fail(LC_ERR_INVALID_ARGUMENT,
                std::string(name) + ": offset " + std::to_string(v.offset) + " beyond buffer capacity " +
                    std::to_string(capacity));
  }
  uint64_t last;
  if (!max_index(v, &last)) return fail(LC_ERR_INVALID_ARGUMENT, std::string(name) + ": index overflow in view");
  if (last >= capacity)
    return fail(LC_ERR_INVALID_ARGUMENT, std::string(name) + ": view reaches element " + std::to_string(last) +
                                             ", buffer holds " + std::to_string(capacity));
  return LC_OK;
}

bool may_overlap(const lc_view& a, const lc_view& b) {
  if (a.data != b.data) return false;
  uint64_t la, lb;
  if (is_empty(a) || is_empty(b)) return false;
  if (!max_index(a, &la) || !max_index(b, &lb)) return true;
  uint64_t a0 = a.offset * dtype_size(a.dtype), a1 = (la + 1) * dtype_size(a.dtype);
  uint64_t b0 = b.offset * dtype_size(b.dtype), b1 = (lb + 1) * dtype_size(b.dtype);
  return a0 < b1 && b0 < a1;
}

bool same_view(const lc_view& a, const lc_view& b) {
  if (a.data != b.data || a.offset != b.offset || a.rank != b.rank) return false;
  for (int d = 0; d < a.rank; d++)
    if (a.shape[d] != b.shape[d] || a.strides[d] != b.strides[d]) return false;
  return true;
}

bool is_injective(const lc_view& v) {
  std::vector<std::pair<uint64_t, uint64_t>> axes;  // (stride, extent)
  for (int d = 0; d < v.rank; d++)
    if (v.shape[d] > 1) axes.push_back({v.strides[d], v.shape[d]});
  std::sort(axes.begin(), axes.end());
  uint64_t max_off = 0;
  for (auto& [stride, extent] : axes) {
    if (stride <= max_off) return false;
    uint64_t step;
    if (__builtin_mul_overflow(stride, extent - 1, &step)) return false;
    if (__builtin_add_overflow(max_off, step, &max_off)) return false;
  }
  return true;
}

bool packed_layout(const lc_view& v) {
  if (v.offset != 0) return false;
  uint64_t stride = 1;
  for (int d = v.rank - 1; d >= 0; d--) {
    if (v.strides[d] != stride) return false;
    stride *= v.shape[d];
  }
  return true;
}

bool is_contiguous(const lc_view& v) {
  uint64_t expect = 1;
  for (int d = v.rank - 1; d >= 0; d--) {
    if (v.shape[d] <= 1) continue;
    if (v.strides[d] != expect) return false;
    if (__builtin_mul_overflow(expect, v.shape[d], &expect)) return false;
  }
  return true;
}

void row_major_strides(const uint64_t* shape, int rank, uint64_t* strides) {
  uint64_t s = 1;
  for (int d = rank - 1; d >= 0; d--) {
    strides[d] = s;
    s *= shape[d];
  }
}

void coalesce(const uint64_t* shape, const uint64_t* strides, int rank, std::vector<uint64_t>* out_shape,
              std::vector<uint64_t>* out_strides) {
  out_shape->clear();
  out_strides->clear();
  for (int d = 0; d < rank; d++) {
    uint64_t n = shape[d], s = strides[d];
    if (n == 1) continue;
    if (!out_shape->empty()) {
      uint64_t prod;
      if (!__builtin_mul_overflow(s, n, &prod) && prod == out_strides->back()) {
        out_shape->back() *= n;
        out_strides->back() = s;
        continue;
      }
    }
    out_shape->push_back(n);
    out_strides->push_back(s);
  }
  if (out_shape->empty()) {
    out_shape->push_back(1);
    out_strides->push_back(1);
  }
}

}  // namespace lc

using namespace lc;

extern "C" {

const char* lc_last_error(void) { return g_last_error.c_str(); }

lc_status lc_context_create(int device, lc_context** out) {
  if (out == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null output pointer");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count <= device || device < 0) {
    cudaGetLastError();
    return fail(LC_ERR_NO_DEVICE, "no CUDA device " + std::to_string(device));
  }
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(LC_ERR_NO_DEVICE, "device " + std::to_string(device) + " is sm_" + std::to_string(prop.major) +
                                      std::to_string(prop.minor) + "; this library is built for sm_100a");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  auto* ctx = new lc_context();
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "cudaStreamCreate");
  }
  e = cudaMalloc(&ctx->d_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_error, 0, sizeof(int), ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return cuda_fail(e, "device error word");
  }
  // Keep freed scratch cached in the pool instead of returning it to the driver.
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  *out = ctx;
  return LC_OK;
}

lc_status lc_context_destroy(lc_context* ctx) {
  if (ctx == nullptr) return LC_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->split_part) cudaFree(ctx->split_part);
  if (ctx->split_cnt) cudaFree(ctx->split_cnt);
  if (ctx->chain_cnt) cudaFree(ctx->chain_cnt);
  cudaFree(ctx->d_error);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return LC_OK;
}

void* lc_context_stream(lc_context* ctx) { return ctx ? ctx->stream : nullptr; }

lc_status lc_sync(lc_context* ctx, void* stream) {
  if (ctx == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null context");
  cudaError_t e = cudaStreamSynchronize(stream_of(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int flag = 0;
  e = cudaMemcpyAsync(&flag, ctx->d_error, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (flag != 0) {
    cudaMemsetAsync(ctx->d_error, 0, sizeof(int), ctx->stream);
    // a launch that gave up may have left split-K arrival counters raised
    if (ctx->split_cnt) cudaMemsetAsync(ctx->split_cnt, 0, ctx->split_cnt_n * sizeof(int), ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    return fail(LC_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait ran out; its output is not valid");
  }
  return LC_OK;
}

uint64_t lc_debug_launches(lc_context* ctx) { return ctx ? ctx->launches.load() : 0; }

const char* lc_debug_launch_name(lc_context* ctx, uint64_t index) {
  if (ctx == nullptr) return nullptr;
  uint64_t n = ctx->launches.load();
  if (index >= n || n - index > kLaunchRing) return nullptr;
  std::lock_guard<std::mutex> g(ctx->names_mu);
  return ctx->names[index % kLaunchRing];
}

lc_status lc_view_validate(const lc_view* v) {
  if (v == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null view");
  return validate(*v, "view");
}

lc_status lc_permute_view(const lc_view* v, const int32_t* perm, int32_t n, lc_view* out) {
  if (v == nullptr || out == nullptr || (perm == nullptr && n > 0))
    return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  int rank = v->rank;
  if (rank < 0 || rank > LC_MAX_RANK) return fail(LC_ERR_INVALID_ARGUMENT, "rank outside 0..8");
  bool seen[LC_MAX_RANK] = {false};
  bool ok = n == rank;
  for (int i = 0; ok && i < n; i++) {
    if (perm[i] < 0 || perm[i] >= rank || seen[perm[i]]) ok = false;
    else seen[perm[i]] = true;
  }
  if (!ok) {
    std::string p = "[";
    for (int i = 0; i < n; i++) p += (i ? ", " : "") + std::to_string(perm[i]);
    return fail(LC_ERR_INVALID_ARGUMENT, p + "] is not a permutation of 0.." + std::to_string(rank));
  }
  lc_view r = *v;
  for (int i = 0; i < rank; i++) {
    r.shape[i] = v->shape[perm[i]];
    r.strides[i] = v->strides[perm[i]];
  }
  *out = r;
  return LC_OK;
}

lc_status lc_slice(const lc_view* v, const uint64_t* starts, const uint64_t* ends, int32_t n, lc_view* out) {
  if (v == nullptr || out == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  lc_status st = validate(*v, "view");
  if (st) return st;
  if (n != v->rank)
    return fail(LC_ERR_INVALID_ARGUMENT,
                "slice expected " + std::to_string(v->rank) + " ranges, got " + std::to_string(n));
  lc_view r = *v;
  uint64_t offset = v->offset;
  for (int d = 0; d < n; d++) {
    if (starts[d] > ends[d]) return fail(LC_ERR_INVALID_ARGUMENT, "inverted range on axis " + std::to_string(d));
    if (ends[d] > v->shape[d])
      return fail(LC_ERR_INVALID_ARGUMENT, "range exceeds extent " + std::to_string(v->shape[d]) + " on axis " +
                                               std::to_string(d));
    uint64_t step;
    if (__builtin_mul_overflow(starts[d], v->strides[d], &step) || __builtin_add_overflow(offset, step, &offset))
      return fail(LC_ERR_INVALID_ARGUMENT, "slice offset overflow on axis " + std::to_string(d));
    r.shape[d] = ends[d] - starts[d];
  }
  r.offset = offset;
  st = validate(r, "slice");
  if (st) return st;
  *out = r;
  return LC_OK;
}

}  // extern "C"
