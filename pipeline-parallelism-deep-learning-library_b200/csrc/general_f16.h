// general_f16.h -- the f16 contraction kernel's geometry (general_f16.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/linalg_b200.h"

namespace lc {

// One index group (batch, M, N or K) as its axes, outermost first: index i of the group is the
// mixed-radix number over ext[], and operand w's element offset for it is sum digit * st[w][axis]
// (w: 0 = A, 1 = B, 2 = C; strides of operands the group does not index are unused).
struct GenGroup {
  int32_t n = 0;
  uint64_t ext[LC_MAX_RANK] = {};
  int64_t st[3][LC_MAX_RANK] = {};
};

struct GenParams {
  uint64_t m = 0, n = 0, k = 0, batch = 1;
  GenGroup gb, gm, gn, gk;
  const uint16_t* a = nullptr;
  const uint16_t* b = nullptr;
  uint16_t* c = nullptr;
  uint64_t a_off = 0, b_off = 0, c_off = 0;
  float alpha = 1.0f, beta = 0.0f;
};

// The f16 product C = alpha * A B + beta * C with one rounding per output, or (fill) the scale
// C = beta * C rounded once / C = 0.
lc_status general_f16_run(lc_context* ctx, cudaStream_t s, const GenParams& p, bool fill);

}  // namespace lc
