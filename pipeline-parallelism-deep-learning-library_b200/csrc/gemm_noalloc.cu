// gemm_noalloc.cu -- lc_encode_gemm with no device allocation.
//
// Who needs it: a caller that must not allocate device memory while it runs, for example a
// serving or training process that reserves the card's memory up front (a pool grown in the
// middle of a step can fail with out-of-memory), or a latency-bound loop where growing a
// stream-ordered pool, or a cudaMalloc/cudaFree, would stall it.  lc_encode_gemm takes its
// split-K scratch from the context (grown with cudaMalloc on first need) or from the device's
// stream-ordered pool; this entry point takes it from the fixed arrays below instead, and
// refuses what does not fit.
//
// The scratch is one pair of arrays per device, shared by every context, stream and thread of
// the process: two calls whose kernels may run at the same time race on it and give wrong
// results.  Callers serialise them (one stream, or events between streams).
#include <cuda_runtime.h>

#include <mutex>

#include "gemm.h"
#include "internal.h"

namespace {

constexpr int kMaxDevices = 64;
// 16 MiB of split-K partial sums (a [splits][batch][M][N] f32 array; a one-wave split of 148
// 128 x 128 tiles takes 9.25 MiB) and one arrival counter per (batch, output tile, epilogue warp)
// for the in-kernel split-K fixup.
constexpr size_t kPartFloats = size_t(4) << 20;
constexpr size_t kCounters = 8192;

static __device__ __align__(256) float g_noalloc_part[kPartFloats];
static __device__ __align__(256) int g_noalloc_cnt[kCounters];

struct DeviceScratch {
  float* part = nullptr;
  int* cnt = nullptr;
};

std::mutex g_mu;
DeviceScratch g_scratch[kMaxDevices];

// Device addresses of the arrays on `device`, looked up once per device.  With lazy module
// loading (CUDA's default) the first lookup also loads this file's module on the device, which
// is when the arrays' memory is reserved there.
lc_status scratch_of(int device, DeviceScratch* out) {
  if (device < 0 || device >= kMaxDevices) return lc::fail(LC_ERR_INVALID_ARGUMENT, "device ordinal out of range");
  std::lock_guard<std::mutex> g(g_mu);
  DeviceScratch& d = g_scratch[device];
  if (d.part == nullptr) {
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess && prev != device) e = cudaSetDevice(device);
    void* part = nullptr;
    void* cnt = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&part, g_noalloc_part);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&cnt, g_noalloc_cnt);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return lc::cuda_fail(e, "cudaGetSymbolAddress(split-K scratch)");
    d.part = static_cast<float*>(part);
    d.cnt = static_cast<int*>(cnt);
  }
  *out = d;
  return LC_OK;
}

}  // namespace

extern "C" {

lc_status lc_encode_gemm_noalloc(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b,
                                 float beta, const lc_view* c) {
  if (ctx == nullptr) return lc::fail(LC_ERR_INVALID_ARGUMENT, "null context");
  DeviceScratch d;
  lc_status st = scratch_of(ctx->device, &d);
  if (st) return st;
  return lc::gemm_fixed_scratch(ctx, stream, alpha, a, b, beta, c, d.part, kPartFloats * sizeof(float), d.cnt,
                                kCounters);
}

}  // extern "C"
