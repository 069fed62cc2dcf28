// gemm.h -- internal interface between the contraction planner and the tensor-core GEMM.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/linalg_b200.h"

namespace lc {

// One operand of a batched product, in elements: element (batch b, row mn, depth k) lives at
// data + offset + b*batch_stride + mn*mn_stride + k*k_stride.
struct GemmOperand {
  const void* data = nullptr;
  uint64_t offset = 0;
  uint64_t mn = 0, k = 0, batch = 1;
  int64_t mn_stride = 0, k_stride = 0, batch_stride = 0;
};

struct GemmProblem {
  uint64_t m = 0, n = 0, k = 0, batch = 1;
  int32_t in_dtype = LC_F32;  // A and B element type: f32 (3xTF32), bf16 or f16
  GemmOperand a, b;           // a: rows M, b: rows N
  void* c = nullptr;          // C base
  int32_t c_dtype = LC_F32;
  uint64_t c_offset = 0;
  int64_t c_batch_stride = 0, c_m_stride = 0, c_n_stride = 0;
  float alpha = 1.0f, beta = 0.0f;
  int32_t relu = 0;           // max(x, 0) after alpha/beta
  int32_t splits_hint = 0;    // 0 = choose
  int32_t bn_hint = 0;        // 0 = choose; 64, 128 or 256 fixes the tile width (16-bit inputs only)
  int32_t swap_hint = 0;      // 0 = choose; 1 = compute C^T = B^T A^T; -1 = never
  int32_t reserve_sms = 0;    // leave this many SMs free (for concurrent communication kernels)
  // Fused epilogues (the training step):
  //   epi 0  C = alpha*acc + beta*C (+ReLU)
  //   epi 1  C = alpha*acc where aux[idx] > 0, else +0  (aux: bf16 with C's layout; the ReLU mask)
  //   epi 2  master[idx] = master[idx] - lr*(alpha*acc); aux2[idx] = bf16(master[idx])
  //          (aux: f32 master weights, aux2: bf16 compute copy, both with C's layout; C unused)
  int32_t epi = 0;
  const void* aux = nullptr;
  void* aux2 = nullptr;
  float lr = 0.0f;
  // Caller-owned split-K scratch (lc_encode_gemm_noalloc): when fixed_part is set, gemm_run takes
  // the partial sums and arrival counters from here, allocates nothing, zeroes the counters it
  // will use, and refuses a split that does not fit.  Null: the context's scratch or the pool.
  float* fixed_part = nullptr;
  size_t fixed_part_bytes = 0;
  int* fixed_cnt = nullptr;
  size_t fixed_cnt_n = 0;
};

// 0 = K-major, 1 = MN-major, -1 = neither (stage it first).  K-major wins when both apply.
inline int operand_major(const GemmOperand& o) {
  if (o.k_stride == 1) return 0;
  if (o.mn_stride == 1) return 1;
  if (o.k == 1) return 0;
  if (o.mn == 1) return 1;
  return -1;
}

// True when TMA can read the operand in place (16-byte aligned start and strides).
bool tma_operand_ok(const GemmOperand& o, int in_dtype);

// Launches the tensor-core GEMM (plus the split-K reduce when it splits).  Operands must pass
// tma_operand_ok.  With dry_run only `plan` is filled.
lc_status gemm_run(lc_context* ctx, cudaStream_t s, const GemmProblem& p, lc_contract_plan* plan, bool dry_run);

// A chain of dependent skinny products (product l + 1 reads what product l writes) in one
// cooperative launch whose CTAs stay resident across the chain.  Each product must plan as a
// 2-way split run by CTA pairs with BN = 64 and all must share one epilogue; otherwise nothing
// is launched and *chained is false (the caller runs the products one by one).  `a_stable`:
// no kernel that may still be running writes any A operand (the weights), so the next
// product's A tiles load ahead of the previous product's completion.  Results are bit-identical
// to launching the products one at a time with gemm_run.
// `max_clusters` (> 0) caps the CTA pairs, leaving the rest of the SMs to work on another
// stream (each pair then takes several tiles of a product).
// The tile width, split count and orientation gemm_run would choose for `pr` (no launch, no
// allocation), the orientation as 1 (C^T = B^T A^T) or -1.  A product over more rows that keeps
// the split count and orientation keeps every output element's k order, split and pair sum; the
// pipeline's grouping test finds the results bit-equal with 64- and 128-wide tiles.
lc_status gemm_plan_shape(lc_context* ctx, const GemmProblem& pr, int32_t* bn, int32_t* splits, int32_t* swap);

lc_status gemm_chain_run(lc_context* ctx, cudaStream_t s, const GemmProblem* probs, int n, bool a_stable,
                         int max_clusters, bool* chained);

// lc_encode_gemm's planning and launch with split-K scratch supplied by the caller: refuses
// products whose operands would need staging copies, or whose split does not fit the scratch.
lc_status gemm_fixed_scratch(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b, float beta,
                             const lc_view* c, float* part, size_t part_bytes, int* cnt, size_t cnt_n);

// C = beta * C, or zeros when beta == 0 (alpha == 0 or K == 0).
lc_status gemm_fill(lc_context* ctx, cudaStream_t s, const GemmProblem& p);

}  // namespace lc
