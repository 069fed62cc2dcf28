// schedule.cpp -- 1F1B order, layer placement and the LNGL wire header (host only).
//
// crates/schedule/src/lib.rs:15-35 (`local_order`), crates/pipeline/src/lib.rs:27-40
// (`contiguous_placement`) and crates/core/src/lib.rs:298-412 (wire header) restated in C++.
// The NCCL data plane sends raw device tiles whose shapes both ranks know, so the wire header
// is only used by host-side transports and tests.
#include <cstring>
#include <string>

#include "internal.h"

using namespace lc;

namespace {
uint32_t tag_of(lc_dtype d) { return d == LC_F32 ? 1u : d == LC_F16 ? 2u : d == LC_BF16 ? 3u : 0u; }
uint64_t size_of_tag(uint32_t t) { return t == 1 ? 4 : (t == 2 || t == 3) ? 2 : 0; }
uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
void wr32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; i++) p[i] = (uint8_t)(v >> (8 * i));
}
}  // namespace

extern "C" {

lc_status lc_local_order(uint64_t stages, uint64_t rank, uint64_t microbatches, int64_t* ops, uint64_t capacity,
                         uint64_t* count) {
  if (stages == 0 || rank >= stages || microbatches == 0 || microbatches > 0xffffffffull)
    return fail(LC_ERR_SCHEDULE, "stages, rank or microbatches out of range");
  if (ops == nullptr || count == nullptr || capacity < 2 * microbatches)
    return fail(LC_ERR_INVALID_ARGUMENT, "order buffer too small");
  const uint64_t m = microbatches, w = stages - rank - 1;
  const uint64_t warmup = w < m ? w : m, steady = m - warmup;
  uint64_t n = 0;
  for (uint64_t i = 0; i < warmup; i++) ops[n++] = (int64_t)i + 1;
  for (uint64_t i = 0; i < steady; i++) {
    ops[n++] = (int64_t)(warmup + i) + 1;
    ops[n++] = -((int64_t)i + 1);
  }
  for (uint64_t i = steady; i < m; i++) ops[n++] = -((int64_t)i + 1);
  *count = n;
  return LC_OK;
}

lc_status lc_contiguous_placement(uint64_t layers, uint64_t stages, uint64_t* owners) {
  if (stages == 0 || layers == 0 || stages > layers) return fail(LC_ERR_SCHEDULE, "layers and stages out of range");
  if (owners == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null owners");
  const uint64_t base = layers / stages, extra = layers % stages;
  uint64_t n = 0;
  for (uint64_t r = 0; r < stages; r++)
    for (uint64_t i = 0; i < base + (r < extra ? 1 : 0); i++) owners[n++] = r;
  return LC_OK;
}

lc_status lc_wire_write_header(lc_dtype dtype, const uint64_t* shape, uint32_t ndim, uint8_t out[48],
                               uint64_t* header_len) {
  if (ndim > 8) return fail(LC_ERR_WIRE, "more than 8 extents");
  const uint32_t tag = tag_of(dtype);
  if (tag == 0) return fail(LC_ERR_DTYPE, "wire dtypes are f32, f16 and bf16");
  uint64_t numel = 1;
  for (uint32_t i = 0; i < ndim; i++) {
    if (shape[i] > 0xffffffffull) return fail(LC_ERR_SHAPE, "extent above u32::MAX");
    if (__builtin_mul_overflow(numel, shape[i], &numel)) return fail(LC_ERR_SHAPE, "element count overflows");
  }
  uint64_t bytes;
  if (__builtin_mul_overflow(numel, size_of_tag(tag), &bytes)) return fail(LC_ERR_SHAPE, "byte count overflows");
  memcpy(out, "LNGL", 4);
  wr32(out + 4, 1);
  wr32(out + 8, tag);
  wr32(out + 12, ndim);
  for (uint32_t i = 0; i < ndim; i++) wr32(out + 16 + 4 * i, (uint32_t)shape[i]);
  *header_len = 16 + 4 * (uint64_t)ndim;
  return LC_OK;
}

lc_status lc_wire_parse_header(const uint8_t* bytes, uint64_t len, lc_dtype* dtype, uint64_t shape[8], uint32_t* ndim,
                               uint64_t* payload_offset) {
  if (bytes == nullptr && len > 0) return fail(LC_ERR_INVALID_ARGUMENT, "null bytes");
  if (len < 16 || memcmp(bytes, "LNGL", 4) != 0) return fail(LC_ERR_WIRE, "bad magic or short message");
  if (rd32(bytes + 4) != 1) return fail(LC_ERR_WIRE, "unsupported wire version");
  const uint32_t tag = rd32(bytes + 8);
  if (size_of_tag(tag) == 0) return fail(LC_ERR_WIRE, "unknown dtype tag");
  const uint32_t nd = rd32(bytes + 12);
  if (nd > 8) return fail(LC_ERR_WIRE, "more than 8 extents");
  const uint64_t header = 16 + 4 * (uint64_t)nd;
  if (len < header) return fail(LC_ERR_WIRE, "truncated extents");
  uint64_t numel = 1;
  for (uint32_t i = 0; i < nd; i++) {
    shape[i] = rd32(bytes + 16 + 4 * i);
    if (__builtin_mul_overflow(numel, shape[i], &numel)) return fail(LC_ERR_SHAPE, "element count overflows");
  }
  uint64_t nbytes;
  if (__builtin_mul_overflow(numel, size_of_tag(tag), &nbytes)) return fail(LC_ERR_SHAPE, "byte count overflows");
  if (len - header != nbytes) return fail(LC_ERR_WIRE, "payload length does not match the shape");
  *dtype = tag == 1 ? LC_F32 : tag == 2 ? LC_F16 : LC_BF16;
  *ndim = nd;
  *payload_offset = header;
  return LC_OK;
}

}  // extern "C"
