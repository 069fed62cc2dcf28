// internal.h -- host-side shared state and helpers of the linalg_b200 library.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/linalg_b200.h"

struct lc_context {
  int device = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;
  int* d_error = nullptr;  // device error word (bit 0: a bounded wait ran out)
  std::atomic<uint64_t> launches{0};
  std::mutex names_mu;
  std::vector<const char*> names;  // ring of the most recent launch names
  // Split-K scratch reused by every GEMM launched on the context's own stream (stream order makes
  // reuse safe): partial tiles, and arrival counters that each launch leaves at zero again.
  void* split_part = nullptr;
  size_t split_part_bytes = 0;
  int* split_cnt = nullptr;
  size_t split_cnt_n = 0;
  // Per-product completion counters of GEMM chain launches (zeroed before each chain), one
  // block of counters per stream that launches chains.
  int* chain_cnt = nullptr;
  void* chain_stream[8] = {};
};

constexpr int kChainStreams = 8;

namespace lc {

// Thread-local error message; returns `code` so `return fail(...)` reads naturally.
lc_status fail(lc_status code, const std::string& msg);
lc_status cuda_fail(cudaError_t e, const char* what);

// Records one kernel launch on the context (name must be a string literal).
void record_launch(lc_context* ctx, const char* name);

// Resolves a NULL stream to the context stream.
inline cudaStream_t stream_of(lc_context* ctx, void* stream) {
  return stream != nullptr ? static_cast<cudaStream_t>(stream) : ctx->stream;
}

// Stream-ordered scratch from the device's default memory pool (kept cached after release).
lc_status scratch_alloc(lc_context* ctx, cudaStream_t s, size_t bytes, void** out);
void scratch_free(void* p, cudaStream_t s);

size_t dtype_size(int32_t dtype);
bool dtype_known(int32_t dtype);

// ---- views ----------------------------------------------------------------------------------

uint64_t numel(const lc_view& v);
bool is_empty(const lc_view& v);
// Largest reachable element index (offset + sum (n-1)*s); false on overflow or empty view.
bool max_index(const lc_view& v, uint64_t* last);
// src/abi.rs:145-177 `validate`.
lc_status validate(const lc_view& v, const char* name);
// src/abi.rs:194-204 `may_overlap`: same buffer and intersecting byte ranges.
bool may_overlap(const lc_view& a, const lc_view& b);
// Same buffer, offset, shape and strides.
bool same_view(const lc_view& a, const lc_view& b);
// src/ops/sqrt.rs:199-226 `is_injective`: distinct multi-indices land on distinct elements.
bool is_injective(const lc_view& v);
// Row-major contiguous at offset 0 (crates/cpu/src/lib.rs:733-746 `packed_layout`).
bool packed_layout(const lc_view& v);
// Logical element i lives at offset + i (src/ops/slicing.rs:189-208 `is_contiguous`).
bool is_contiguous(const lc_view& v);
// Row-major strides of a shape.
void row_major_strides(const uint64_t* shape, int rank, uint64_t* strides);

// src/ops/permutation.rs:110-132 `coalesce`: drop unit axes, merge axes contiguous in the source.
void coalesce(const uint64_t* shape, const uint64_t* strides, int rank, std::vector<uint64_t>* out_shape,
              std::vector<uint64_t>* out_strides);

// ---- kernel entry points used across translation units -------------------------------------

// Elementwise/strided gather copy of raw elements (elem_bytes in {1,2,4,8,16}):
// dst[dst_off + sum idx*dst_strides] = src[src_off + sum idx*src_strides]; conj flips the sign bit
// of the second 4-byte word of 8-byte elements.  Picks the tiled transpose, the row-vector copy or
// the scalar copy.  Views are assumed validated and non-overlapping.
lc_status launch_strided_copy(lc_context* ctx, cudaStream_t s, const void* src, uint64_t src_off,
                              void* dst, uint64_t dst_off, int rank, const uint64_t* shape,
                              const uint64_t* src_strides, const uint64_t* dst_strides, size_t elem_bytes,
                              bool conj);

}  // namespace lc
