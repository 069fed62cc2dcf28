// contraction.cpp -- planner of C = alpha*A*B + beta*C over einsum labels and batched GEMM views.
//
// Restates src/ops/contraction.rs's planning rules:
//   labels -> roles (`groups_from_labels`, :380-442): in A,B,C batch; A,C -> M; B,C -> N;
//             A,B -> K; a label in C only, or in one operand, is an error; extents must agree;
//   group order: batch, M and N follow C's labels, K follows A's labels;
//   alias rules (`check_destination_alias`, :637-662): C may not write an element twice and may
//             not overlap an input it reads, except the in-place scale C = alpha*C*s;
//   scalar rules: beta == 0 never reads C, alpha == 0 never reads A or B, K == 0 gives beta*C,
//             an empty batch/M/N launches nothing (`plan_merged`, :811-867).
// The B200 plan differs in how it executes, not in what it computes:
//   - each operand's groups are merged on that operand's own strides (adjacent axes contiguous
//     in that operand fold together), so a layout that is contiguous for A but not for C stages
//     only C;
//   - an operand whose group still has several strides, or whose strides TMA cannot address
//     (16-byte rules), is first materialised into a dense K-major scratch copy by the strided
//     copy engine (the "permute -> GEMM" path); a C that is not single-stride is computed into
//     a dense scratch C and packed back;
//   - split-K is chosen for the 148-SM part (units = tiles x batch below the SM count), with
//     partials reduced in split order (deterministic).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <unordered_set>
#include <vector>

#include "gemm.h"
#include "general_f16.h"
#include "internal.h"

namespace {

using namespace lc;

struct Axis {
  uint64_t extent;
  bool in_a, in_b, in_c;
  uint64_t sa, sb, sc;
};

enum Role { kBatch, kM, kN, kK };

struct Groups {
  std::vector<Axis> batch, m, n, k;
};

struct Merged1 {  // one operand's view of one group after merging
  std::vector<std::pair<uint64_t, uint64_t>> axes;  // (extent, stride), outermost first
};

// Drops extent-1 axes; folds an axis into its outer neighbour when contiguous in this operand.
Merged1 merge_for(const std::vector<Axis>& axes, int which) {
  Merged1 r;
  for (const Axis& ax : axes) {
    if (ax.extent == 1) continue;
    uint64_t st = which == 0 ? ax.sa : which == 1 ? ax.sb : ax.sc;
    if (!r.axes.empty()) {
      auto& prev = r.axes.back();
      uint64_t prod;
      if (!__builtin_mul_overflow(ax.extent, st, &prod) && prev.second == prod) {
        prev.first *= ax.extent;
        prev.second = st;
        continue;
      }
    }
    r.axes.push_back({ax.extent, st});
  }
  return r;
}

uint64_t product(const std::vector<Axis>& axes) {
  uint64_t p = 1;
  for (const Axis& a : axes) p *= a.extent;
  return p;
}

lc_status parse_labels(const char* labels, int rank, std::vector<char>* out) {
  if (labels == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null labels");
  size_t n = strlen(labels);
  if ((int)n != rank)
    return fail(LC_ERR_INVALID_ARGUMENT,
                "label count " + std::to_string(n) + " does not match rank " + std::to_string(rank));
  out->assign(labels, labels + n);
  for (size_t i = 0; i < n; i++)
    for (size_t j = 0; j < i; j++)
      if ((*out)[i] == (*out)[j]) return fail(LC_ERR_INVALID_ARGUMENT, std::string("repeated label '") + (*out)[i] + "'");
  return LC_OK;
}

lc_status groups_from_labels(const lc_view& a, const std::vector<char>& la, const lc_view& b,
                             const std::vector<char>& lb, const lc_view& c, const std::vector<char>& lc_,
                             Groups* g) {
  std::vector<char> order;
  for (auto* v : {&la, &lb, &lc_})
    for (char ch : *v)
      if (std::find(order.begin(), order.end(), ch) == order.end()) order.push_back(ch);
  struct Info {
    char ch;
    Role role;
    Axis axis;
  };
  std::vector<Info> infos;
  auto find = [](const std::vector<char>& l, char ch) -> int {
    auto it = std::find(l.begin(), l.end(), ch);
    return it == l.end() ? -1 : (int)(it - l.begin());
  };
  for (char ch : order) {
    int fa = find(la, ch), fb = find(lb, ch), fc = find(lc_, ch);
    Role role;
    if (fa >= 0 && fb >= 0 && fc >= 0) role = kBatch;
    else if (fa >= 0 && fb < 0 && fc >= 0) role = kM;
    else if (fa < 0 && fb >= 0 && fc >= 0) role = kN;
    else if (fa >= 0 && fb >= 0 && fc < 0) role = kK;
    else if (fa < 0 && fb < 0 && fc >= 0) return fail(LC_ERR_INVALID_ARGUMENT, std::string("label '") + ch + "' appears only in C");
    else return fail(LC_ERR_INVALID_ARGUMENT, std::string("label '") + ch + "' appears once");
    uint64_t extent = 0;
    bool have = false;
    for (auto [pos, view] : {std::pair<int, const lc_view*>{fa, &a}, {fb, &b}, {fc, &c}}) {
      if (pos < 0) continue;
      if (!have) {
        extent = view->shape[pos];
        have = true;
      } else if (extent != view->shape[pos]) {
        return fail(LC_ERR_INVALID_ARGUMENT, std::string("extent mismatch for label '") + ch + "'");
      }
    }
    Axis ax{extent, fa >= 0, fb >= 0, fc >= 0, fa >= 0 ? a.strides[fa] : 0, fb >= 0 ? b.strides[fb] : 0,
            fc >= 0 ? c.strides[fc] : 0};
    infos.push_back({ch, role, ax});
  }
  auto take = [&](const std::vector<char>& labels, Role role) {
    std::vector<Axis> out;
    for (char ch : labels)
      for (const Info& in : infos)
        if (in.ch == ch && in.role == role) out.push_back(in.axis);
    return out;
  };
  g->batch = take(lc_, kBatch);
  g->m = take(lc_, kM);
  g->n = take(lc_, kN);
  g->k = take(la, kK);
  return LC_OK;
}

// src/ops/contraction.rs:444-494 `groups_from_gemm`.
lc_status groups_from_gemm(const lc_view& a, const lc_view& b, const lc_view& c, Groups* g) {
  if (a.rank < 2 || b.rank < 2 || c.rank < 2) return fail(LC_ERR_INVALID_ARGUMENT, "rank below 2");
  if (a.rank != b.rank || b.rank != c.rank) return fail(LC_ERR_INVALID_ARGUMENT, "ranks differ");
  int r = a.rank;
  g->batch.clear();
  for (int d = 0; d < r - 2; d++) {
    if (a.shape[d] != b.shape[d] || b.shape[d] != c.shape[d]) return fail(LC_ERR_INVALID_ARGUMENT, "batch extents differ");
    g->batch.push_back({a.shape[d], true, true, true, a.strides[d], b.strides[d], c.strides[d]});
  }
  uint64_t m = a.shape[r - 2], ka = a.shape[r - 1], kb = b.shape[r - 2], n = b.shape[r - 1];
  if (m != c.shape[r - 2] || n != c.shape[r - 1] || ka != kb) return fail(LC_ERR_INVALID_ARGUMENT, "inner extents differ");
  g->m = {{m, true, false, true, a.strides[r - 2], 0, c.strides[r - 2]}};
  g->n = {{n, false, true, true, 0, b.strides[r - 1], c.strides[r - 1]}};
  g->k = {{ka, true, true, false, a.strides[r - 1], b.strides[r - 2], 0}};
  return LC_OK;
}

// ---- alias analysis (src/ops/contraction.rs:496-662) -------------------------------------------

// Extent>1 axes sorted by stride when they form a unique mixed-radix address.
bool decodable(const lc_view& v, std::vector<std::pair<uint64_t, uint64_t>>* axes) {
  axes->clear();
  for (int d = 0; d < v.rank; d++)
    if (v.shape[d] > 1) axes->push_back({v.shape[d], v.strides[d]});
  std::sort(axes->begin(), axes->end(), [](auto& x, auto& y) { return x.second < y.second; });
  for (auto& ax : *axes)
    if (ax.second == 0) return false;
  for (size_t i = 1; i < axes->size(); i++) {
    uint64_t span;
    if (__builtin_mul_overflow((*axes)[i - 1].second, (*axes)[i - 1].first, &span) || (*axes)[i].second < span)
      return false;
  }
  return true;
}

bool contains(const lc_view& v, uint64_t elem, const std::vector<std::pair<uint64_t, uint64_t>>& asc) {
  if (elem < v.offset) return false;
  uint64_t rem = elem - v.offset;
  for (auto it = asc.rbegin(); it != asc.rend(); ++it) {
    uint64_t coord = rem / it->second;
    if (coord >= it->first) return false;
    rem -= coord * it->second;
  }
  return rem == 0;
}

template <typename F>
void for_each_index(const lc_view& v, F visit) {
  if (is_empty(v)) return;
  if (v.rank == 0) {
    visit(v.offset);
    return;
  }
  uint64_t idx[LC_MAX_RANK] = {0};
  for (;;) {
    uint64_t e = v.offset;
    for (int d = 0; d < v.rank; d++) e += idx[d] * v.strides[d];
    visit(e);
    int ax = v.rank - 1;
    for (;;) {
      if (++idx[ax] < v.shape[ax]) break;
      idx[ax] = 0;
      if (ax == 0) return;
      ax--;
    }
  }
}

constexpr uint64_t kExactLimit = 2000000;

bool range_of(const lc_view& v, uint64_t* lo, uint64_t* hi) {
  uint64_t last;
  if (!max_index(v, &last)) return false;
  *lo = v.offset;
  *hi = last + 1;
  return true;
}

bool shares(const lc_view& a, const lc_view& b) {
  if (a.data != b.data) return false;
  uint64_t a0, a1, b0, b1;
  if (!range_of(a, &a0, &a1) || !range_of(b, &b0, &b1)) return false;
  if (a0 >= b1 || b0 >= a1) return false;
  const lc_view& small = numel(a) <= numel(b) ? a : b;
  const lc_view& large = numel(a) <= numel(b) ? b : a;
  std::vector<std::pair<uint64_t, uint64_t>> axes;
  if (decodable(large, &axes)) {
    bool hit = false;
    for_each_index(small, [&](uint64_t e) { hit = hit || contains(large, e, axes); });
    return hit;
  }
  if (numel(large) > kExactLimit) return true;
  std::unordered_set<uint64_t> seen;
  for_each_index(large, [&](uint64_t e) { seen.insert(e); });
  bool hit = false;
  for_each_index(small, [&](uint64_t e) { hit = hit || seen.count(e) > 0; });
  return hit;
}

bool self_overlaps(const lc_view& v) {
  std::vector<std::pair<uint64_t, uint64_t>> axes;
  if (numel(v) <= 1 || decodable(v, &axes)) return false;
  if (numel(v) > kExactLimit) return true;
  std::unordered_set<uint64_t> seen;
  bool overlap = false;
  for_each_index(v, [&](uint64_t e) { overlap = overlap || !seen.insert(e).second; });
  return overlap;
}

lc_status check_destination_alias(const lc_view& a, const lc_view& b, const lc_view& c, uint64_t m, uint64_t n,
                                  uint64_t k, bool reads_inputs) {
  if (self_overlaps(c)) return fail(LC_ERR_OVERLAP, "C writes the same element more than once");
  if (!reads_inputs) return LC_OK;
  const bool inplace_a = k == 1 && n == 1 && same_view(c, a) && !shares(c, b);
  const bool inplace_b = k == 1 && m == 1 && same_view(c, b) && !shares(c, a);
  if (!inplace_a && (same_view(c, a) || shares(c, a))) return fail(LC_ERR_OVERLAP, "C overlaps A");
  if (!inplace_b && (same_view(c, b) || shares(c, b))) return fail(LC_ERR_OVERLAP, "C overlaps B");
  return LC_OK;
}

// ---- staging -------------------------------------------------------------------------------------

struct Staged {
  void* buf = nullptr;
};

// Builds the operand's view as [batch axes][row axes][depth axes] with its own strides.
void collect(const std::vector<Axis>& axes, int which, std::vector<uint64_t>* shape, std::vector<uint64_t>* strides) {
  for (const Axis& ax : axes) {
    if (ax.extent == 1) continue;
    shape->push_back(ax.extent);
    strides->push_back(which == 0 ? ax.sa : which == 1 ? ax.sb : ax.sc);
  }
}

// Dense row-major strides for [batch..][rows..][depth..] with the depth row padded to `row_len`.
void dense_strides(const std::vector<uint64_t>& shape, size_t nb, size_t nr, uint64_t row_len, uint64_t rows_total,
                   std::vector<uint64_t>* out) {
  out->assign(shape.size(), 0);
  uint64_t s = 1;
  for (size_t i = shape.size(); i-- > nb + nr;) {
    (*out)[i] = s;
    s *= shape[i];
  }
  s = row_len;
  for (size_t i = nb + nr; i-- > nb;) {
    (*out)[i] = s;
    s *= shape[i];
  }
  s = row_len * rows_total;
  for (size_t i = nb; i-- > 0;) {
    (*out)[i] = s;
    s *= shape[i];
  }
}

struct Plan {
  int kind = 0;  // 0 empty, 1 fill, 2 gemm
  GemmProblem prob;
  // f16 with the op API's rounding: the product (or the fill) runs on general_f16_run, reading
  // the operands in place through the groups' strides
  bool f16_general = false;
  Groups groups;
  bool stage_a = false, stage_b = false, stage_c = false;
  // staging geometry
  std::vector<uint64_t> a_shape, a_src, b_shape, b_src, c_shape, c_src;
  size_t a_nb = 0, a_nr = 0, b_nb = 0, b_nr = 0, c_nb = 0, c_nm = 0;
  uint64_t a_row = 0, b_row = 0;
  const lc_view *av = nullptr, *bv = nullptr, *cv = nullptr;
};

bool single(const Merged1& m) { return m.axes.size() <= 1; }
uint64_t stride1(const Merged1& m) { return m.axes.empty() ? 0 : m.axes[0].second; }

lc_status plan_groups(lc_context* ctx, const lc_view& a, const lc_view& b, const lc_view& c, const Groups& g, float alpha,
                      float beta, Plan* plan) {
  const uint64_t bt = product(g.batch), mt = product(g.m), nt = product(g.n), kt = product(g.k);
  plan->av = &a;
  plan->bv = &b;
  plan->cv = &c;
  GemmProblem& pr = plan->prob;
  plan->groups = g;
  pr.m = mt;
  pr.n = nt;
  pr.k = kt;
  pr.batch = bt;
  pr.in_dtype = a.dtype;
  pr.c_dtype = c.dtype;
  pr.alpha = alpha;
  pr.beta = beta;
  if (mt == 0 || nt == 0 || bt == 0) {
    plan->kind = 0;
    return LC_OK;
  }
  const bool reads_inputs = alpha != 0.0f && kt != 0;
  lc_status st = check_destination_alias(a, b, c, mt, nt, kt, reads_inputs);
  if (st) return st;
  // C geometry (needed by both plans)
  Merged1 cb = merge_for(g.batch, 2), cm = merge_for(g.m, 2), cn = merge_for(g.n, 2);
  if (single(cb) && single(cm) && single(cn)) {
    pr.c = c.data;
    pr.c_offset = c.offset;
    pr.c_batch_stride = (int64_t)stride1(cb);
    pr.c_m_stride = (int64_t)stride1(cm);
    pr.c_n_stride = (int64_t)stride1(cn);
    if (cm.axes.empty()) pr.c_m_stride = (int64_t)nt;  // extent-1 group: any stride; keep it aligned-friendly
    if (cn.axes.empty()) pr.c_n_stride = 1;
    if (cb.axes.empty()) pr.c_batch_stride = (int64_t)(mt * nt);
  } else {
    plan->stage_c = true;
    collect(g.batch, 2, &plan->c_shape, &plan->c_src);
    plan->c_nb = plan->c_shape.size();
    collect(g.m, 2, &plan->c_shape, &plan->c_src);
    plan->c_nm = plan->c_shape.size() - plan->c_nb;
    collect(g.n, 2, &plan->c_shape, &plan->c_src);
    pr.c_offset = 0;
    pr.c_batch_stride = (int64_t)(mt * nt);
    pr.c_m_stride = (int64_t)nt;
    pr.c_n_stride = 1;
  }
  if (!reads_inputs) {
    plan->kind = 1;
    return LC_OK;
  }
  plan->kind = 2;
  const size_t es = dtype_size(a.dtype);
  const uint64_t pad = 16 / es;  // elements per 16 bytes
  // A
  Merged1 ab = merge_for(g.batch, 0), am = merge_for(g.m, 0), ak = merge_for(g.k, 0);
  GemmOperand& A = pr.a;
  A.data = a.data;
  A.offset = a.offset;
  A.mn = mt;
  A.k = kt;
  A.batch = bt;
  A.batch_stride = (int64_t)stride1(ab);
  A.mn_stride = (int64_t)stride1(am);
  A.k_stride = (int64_t)stride1(ak);
  if (am.axes.empty()) A.mn_stride = 0;
  if (ak.axes.empty()) A.k_stride = 0;
  if (!(single(ab) && single(am) && single(ak)) || !tma_operand_ok(A, a.dtype)) {
    plan->stage_a = true;
    collect(g.batch, 0, &plan->a_shape, &plan->a_src);
    plan->a_nb = plan->a_shape.size();
    collect(g.m, 0, &plan->a_shape, &plan->a_src);
    plan->a_nr = plan->a_shape.size() - plan->a_nb;
    collect(g.k, 0, &plan->a_shape, &plan->a_src);
    plan->a_row = (kt + pad - 1) / pad * pad;
    A.data = nullptr;
    A.offset = 0;
    A.k_stride = 1;
    A.mn_stride = (int64_t)plan->a_row;
    A.batch_stride = (int64_t)(plan->a_row * mt);
  }
  // B
  Merged1 bb = merge_for(g.batch, 1), bn_ = merge_for(g.n, 1), bk = merge_for(g.k, 1);
  GemmOperand& B = pr.b;
  B.data = b.data;
  B.offset = b.offset;
  B.mn = nt;
  B.k = kt;
  B.batch = bt;
  B.batch_stride = (int64_t)stride1(bb);
  B.mn_stride = (int64_t)stride1(bn_);
  B.k_stride = (int64_t)stride1(bk);
  if (bn_.axes.empty()) B.mn_stride = 0;
  if (bk.axes.empty()) B.k_stride = 0;
  if (!(single(bb) && single(bn_) && single(bk)) || !tma_operand_ok(B, b.dtype)) {
    plan->stage_b = true;
    collect(g.batch, 1, &plan->b_shape, &plan->b_src);
    plan->b_nb = plan->b_shape.size();
    collect(g.n, 1, &plan->b_shape, &plan->b_src);
    plan->b_nr = plan->b_shape.size() - plan->b_nb;
    collect(g.k, 1, &plan->b_shape, &plan->b_src);
    plan->b_row = (kt + pad - 1) / pad * pad;
    B.data = nullptr;
    B.offset = 0;
    B.k_stride = 1;
    B.mn_stride = (int64_t)plan->b_row;
    B.batch_stride = (int64_t)(plan->b_row * nt);
  }
  (void)ctx;
  return LC_OK;
}

lc_status stage_operand(lc_context* ctx, cudaStream_t s, const lc_view& v, const std::vector<uint64_t>& shape,
                        const std::vector<uint64_t>& src_strides, size_t nb, size_t nr, uint64_t row_len, uint64_t rows,
                        uint64_t batch, void** out) {
  const size_t es = dtype_size(v.dtype);
  lc_status st = scratch_alloc(ctx, s, es * row_len * rows * batch, out);
  if (st) return st;
  if (row_len * rows * batch != 0 && row_len > 0) {
    // zero the K padding so nothing uninitialised can reach an accumulator (TMA reads only up to
    // K, but keep the scratch deterministic)
    cudaMemsetAsync(*out, 0, es * row_len * rows * batch, s);
  }
  std::vector<uint64_t> dst;
  dense_strides(shape, nb, nr, row_len, rows, &dst);
  if (shape.empty()) {
    uint64_t one = 1, z = 0;
    return launch_strided_copy(ctx, s, v.data, v.offset, *out, 0, 1, &one, &z, &z, es, false);
  }
  return launch_strided_copy(ctx, s, v.data, v.offset, *out, 0, (int)shape.size(), shape.data(), src_strides.data(),
                             dst.data(), es, false);
}

lc_status execute(lc_context* ctx, cudaStream_t s, Plan& plan, lc_contract_plan* report, bool dry_run) {
  GemmProblem& pr = plan.prob;
  if (report) {
    memset(report, 0, sizeof(*report));
    report->kind = plan.kind;
    report->splits = 1;
    report->batch = pr.batch;
    report->m = pr.m;
    report->n = pr.n;
    report->k = pr.k;
  }
  if (plan.kind == 0) return LC_OK;
  if (plan.f16_general) {
    if (report && plan.kind == 2) report->kind = 5;
    if (dry_run) return LC_OK;
    GenParams gp;
    gp.m = pr.m;
    gp.n = pr.n;
    gp.k = pr.k;
    gp.batch = pr.batch;
    auto fill_group = [](const std::vector<Axis>& axes, GenGroup* out) {
      out->n = 0;
      for (const Axis& ax : axes) {
        out->ext[out->n] = ax.extent;
        out->st[0][out->n] = (int64_t)ax.sa;
        out->st[1][out->n] = (int64_t)ax.sb;
        out->st[2][out->n] = (int64_t)ax.sc;
        out->n++;
      }
    };
    fill_group(plan.groups.batch, &gp.gb);
    fill_group(plan.groups.m, &gp.gm);
    fill_group(plan.groups.n, &gp.gn);
    fill_group(plan.groups.k, &gp.gk);
    gp.a = static_cast<const uint16_t*>(plan.av->data);
    gp.b = static_cast<const uint16_t*>(plan.bv->data);
    gp.c = static_cast<uint16_t*>(plan.cv->data);
    gp.a_off = plan.av->offset;
    gp.b_off = plan.bv->offset;
    gp.c_off = plan.cv->offset;
    gp.alpha = pr.alpha;
    gp.beta = pr.beta;
    return general_f16_run(ctx, s, gp, plan.kind == 1);
  }
  if (dry_run && plan.kind == 1) return LC_OK;
  if (dry_run) {
    GemmProblem q = pr;
    // placeholder pointers for staged operands: staging produces 256-byte aligned dense copies
    static const uint8_t* kAligned = reinterpret_cast<const uint8_t*>(uintptr_t(1) << 20);
    if (plan.stage_a) q.a.data = kAligned;
    if (plan.stage_b) q.b.data = kAligned;
    if (plan.stage_c) q.c = const_cast<uint8_t*>(kAligned);
    lc_status st = gemm_run(ctx, s, q, report, true);
    if (report && (plan.stage_a || plan.stage_b || plan.stage_c)) report->kind = 4;
    return st;
  }
  const lc_view& c = *plan.cv;
  const size_t ces = dtype_size(c.dtype);
  void *sa = nullptr, *sb = nullptr, *sc = nullptr;
  lc_status st = LC_OK;
  std::vector<uint64_t> cdst;
  if (plan.stage_c) {
    st = scratch_alloc(ctx, s, ces * pr.m * pr.n * pr.batch, &sc);
    if (st) return st;
    pr.c = sc;
    dense_strides(plan.c_shape, plan.c_nb, plan.c_nm, pr.n, pr.m, &cdst);
    // the n axes are innermost and dense: dense_strides with row_len = n covers [b][m][n]
    if (pr.beta != 0.0f)
      st = launch_strided_copy(ctx, s, c.data, c.offset, sc, 0, (int)plan.c_shape.size(), plan.c_shape.data(),
                               plan.c_src.data(), cdst.data(), ces, false);
  }
  if (!st && plan.kind == 1) {
    st = gemm_fill(ctx, s, pr);
  } else if (!st) {
    if (plan.stage_a)
      st = stage_operand(ctx, s, *plan.av, plan.a_shape, plan.a_src, plan.a_nb, plan.a_nr, plan.a_row, pr.m, pr.batch,
                         &sa);
    if (!st && plan.stage_b)
      st = stage_operand(ctx, s, *plan.bv, plan.b_shape, plan.b_src, plan.b_nb, plan.b_nr, plan.b_row, pr.n, pr.batch,
                         &sb);
    if (!st) {
      if (sa) pr.a.data = sa;
      if (sb) pr.b.data = sb;
      st = gemm_run(ctx, s, pr, report, false);
      if (report && (plan.stage_a || plan.stage_b || plan.stage_c)) report->kind = 4;
    }
  }
  if (!st && plan.stage_c) {
    std::vector<uint64_t> cd = cdst;
    st = launch_strided_copy(ctx, s, sc, 0, c.data, c.offset, (int)plan.c_shape.size(), plan.c_shape.data(), cd.data(),
                             plan.c_src.data(), ces, false);
  }
  scratch_free(sa, s);
  scratch_free(sb, s);
  scratch_free(sc, s);
  if (!st) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) st = cuda_fail(e, "contraction");
  }
  return st;
}

lc_status check_types(const lc_view& a, const lc_view& b, const lc_view& c) {
  if (a.dtype != b.dtype || a.dtype != c.dtype)
    return fail(LC_ERR_INVALID_ARGUMENT, "A, B and C must share one element type");
  if (a.dtype != LC_F32 && a.dtype != LC_BF16 && a.dtype != LC_F16)
    return fail(LC_ERR_INVALID_ARGUMENT, "contraction element types are f32, f16 and bf16");
  return LC_OK;
}

lc_status prepare(const lc_view* a, const lc_view* b, const lc_view* c) {
  if (a == nullptr || b == nullptr || c == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null view");
  lc_status st = validate(*a, "A");
  if (!st) st = validate(*b, "B");
  if (!st) st = validate(*c, "C");
  if (!st) st = check_types(*a, *b, *c);
  return st;
}

lc_status contract_impl(lc_context* ctx, void* stream, float alpha, const lc_view* a, const char* la,
                        const lc_view* b, const char* lb, float beta, const lc_view* c, const char* lcl,
                        lc_contract_plan* report, bool dry_run) {
  // Planning alone needs no device: without a context it plans for a 148-SM B200.
  static lc_context planning_only;
  if (ctx == nullptr && dry_run) ctx = &planning_only;
  if (ctx == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null context");
  lc_status st = prepare(a, b, c);
  if (st) return st;
  std::vector<char> pa, pb, pc;
  if ((st = parse_labels(la, a->rank, &pa))) return st;
  if ((st = parse_labels(lb, b->rank, &pb))) return st;
  if ((st = parse_labels(lcl, c->rank, &pc))) return st;
  Groups g;
  if ((st = groups_from_labels(*a, pa, *b, pb, *c, pc, &g))) return st;
  Plan plan;
  if ((st = plan_groups(ctx, *a, *b, *c, g, alpha, beta, &plan))) return st;
  plan.f16_general = a->dtype == LC_F16;
  return execute(ctx, stream_of(ctx, stream), plan, report, dry_run);
}

// op_api: the op API's `gemm` (f16 rounds once from a double-float dot); otherwise the Backend
// slot's gemm, whose f16 products run on the tensor cores with f32 accumulation.
lc_status gemm_impl(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b, float beta,
                    const lc_view* c, bool op_api) {
  if (ctx == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null context");
  lc_status st = prepare(a, b, c);
  if (st) return st;
  Groups g;
  if ((st = groups_from_gemm(*a, *b, *c, &g))) return st;
  Plan plan;
  if ((st = plan_groups(ctx, *a, *b, *c, g, alpha, beta, &plan))) return st;
  plan.f16_general = op_api && a->dtype == LC_F16;
  return execute(ctx, stream_of(ctx, stream), plan, nullptr, false);
}

// A fused epilogue's side view must be laid out exactly like C: the epilogue reads and writes it
// at C's element index.
lc_status same_layout_as_c(const lc_view* v, const lc_view& c, int32_t dtype, const char* what) {
  if (v == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, std::string("this epilogue needs ") + what);
  lc_status st = validate(*v, what);
  if (st) return st;
  if (v->dtype != dtype) return fail(LC_ERR_DTYPE, std::string(what) + " has the wrong element type");
  if (v->rank != c.rank || v->offset != c.offset) return fail(LC_ERR_SHAPE, std::string(what) + " must be laid out like C");
  for (int i = 0; i < c.rank; i++)
    if (v->shape[i] != c.shape[i] || (c.shape[i] > 1 && v->strides[i] != c.strides[i]))
      return fail(LC_ERR_SHAPE, std::string(what) + " must be laid out like C");
  return LC_OK;
}

lc_status gemm_fused_impl(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b, float beta,
                          const lc_view* c, const lc_epilogue* e) {
  if (ctx == nullptr || e == nullptr || c == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  // SGD: A and B are 16-bit, C (the master weights) f32; the type checks see a C of the inputs'
  // type with C's geometry
  lc_view c16 = *c;
  if (e->kind == LC_EPI_SGD && a != nullptr) {
    if (c->dtype != LC_F32) return fail(LC_ERR_DTYPE, "the SGD epilogue updates f32 master weights");
    lc_status vs = validate(*c, "C");
    if (vs) return vs;
    c16.dtype = a->dtype;
  }
  lc_status st = prepare(a, b, &c16);
  if (st) return st;
  if (e->kind < LC_EPI_NONE || e->kind > LC_EPI_GELU_BACKWARD) return fail(LC_ERR_INVALID_ARGUMENT, "unknown epilogue kind");
  if (e->tile_n != 0 && e->tile_n != 64 && e->tile_n != 128 && e->tile_n != 256)
    return fail(LC_ERR_INVALID_ARGUMENT, "tile_n is 0, 64, 128 or 256");
  if (e->splits < 0) return fail(LC_ERR_INVALID_ARGUMENT, "negative split count");
  const bool sixteen = a->dtype != LC_F32;
  if ((e->kind == LC_EPI_RELU_MASK || e->kind == LC_EPI_SGD) && !sixteen)
    return fail(LC_ERR_DTYPE, "the mask and SGD epilogues take bf16 or f16 inputs");
  if ((e->kind == LC_EPI_GELU || e->kind == LC_EPI_GELU_BACKWARD) && sixteen)
    return fail(LC_ERR_DTYPE, "the GELU epilogues take f32 operands");
  if (e->kind == LC_EPI_GELU_BACKWARD && beta != 0.0f)
    return fail(LC_ERR_INVALID_ARGUMENT, "the GELU backward epilogue takes beta = 0");
  Groups g;
  if ((st = groups_from_gemm(*a, *b, c16, &g))) return st;
  Plan plan;
  if ((st = plan_groups(ctx, *a, *b, *c, g, alpha, beta, &plan))) return st;
  if (e->kind != LC_EPI_NONE) {
    if (plan.kind != 2) return fail(LC_ERR_INVALID_ARGUMENT, "fused epilogues need alpha != 0 and K > 0");
    if (plan.stage_c)
      return fail(LC_ERR_UNSUPPORTED_LAYOUT, "fused epilogues need C with one stride per index group");
  }
  GemmProblem& pr = plan.prob;
  pr.bn_hint = e->tile_n;
  pr.splits_hint = e->splits;
  pr.swap_hint = e->swap;
  switch (e->kind) {
    case LC_EPI_RELU:
      pr.relu = 1;
      break;
    case LC_EPI_RELU_MASK:
      if ((st = same_layout_as_c(e->aux, *c, LC_BF16, "aux (the ReLU mask source)"))) return st;
      pr.epi = 1;
      pr.aux = e->aux->data;
      break;
    case LC_EPI_SGD:
      if ((st = same_layout_as_c(e->aux2, *c, LC_BF16, "aux2 (the bf16 weight copy)"))) return st;
      if (e->aux2->data == c->data) return fail(LC_ERR_ALIAS, "aux2 shares C's storage");
      pr.epi = 2;
      pr.aux = c->data;
      pr.aux2 = e->aux2->data;
      pr.lr = e->lr;
      pr.c_dtype = LC_F32;
      break;
    case LC_EPI_GELU:
      if (e->aux2 != nullptr) {
        if ((st = same_layout_as_c(e->aux2, *c, LC_F32, "aux2 (the pre-activation output)"))) return st;
        if (e->aux2->data == c->data) return fail(LC_ERR_ALIAS, "aux2 shares C's storage");
        pr.aux2 = e->aux2->data;
      }
      pr.epi = 3;
      break;
    case LC_EPI_GELU_BACKWARD:
      if ((st = same_layout_as_c(e->aux, *c, LC_F32, "aux (the pre-activation)"))) return st;
      pr.epi = 4;
      pr.aux = e->aux->data;
      break;
    default:
      break;
  }
  return execute(ctx, stream_of(ctx, stream), plan, nullptr, false);
}

}  // namespace

namespace lc {

lc_status gemm_fixed_scratch(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b, float beta,
                             const lc_view* c, float* part, size_t part_bytes, int* cnt, size_t cnt_n) {
  if (ctx == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null context");
  lc_status st = prepare(a, b, c);
  if (st) return st;
  Groups g;
  if ((st = groups_from_gemm(*a, *b, *c, &g))) return st;
  Plan plan;
  if ((st = plan_groups(ctx, *a, *b, *c, g, alpha, beta, &plan))) return st;
  plan.f16_general = a->dtype == LC_F16;  // lc_encode_gemm's semantics; it needs no scratch
  if (!plan.f16_general && (plan.stage_a || plan.stage_b || plan.stage_c))
    return fail(LC_ERR_INVALID_ARGUMENT,
                "this product needs staging copies of its operands, which the allocation-free entry point "
                "cannot hold: pass operands with a unit stride and 16-byte aligned starts and strides");
  plan.prob.fixed_part = part;
  plan.prob.fixed_part_bytes = part_bytes;
  plan.prob.fixed_cnt = cnt;
  plan.prob.fixed_cnt_n = cnt_n;
  return execute(ctx, stream_of(ctx, stream), plan, nullptr, false);
}

}  // namespace lc

extern "C" {

lc_status lc_encode_contract(lc_context* ctx, void* stream, float alpha, const lc_view* a, const char* a_labels,
                             const lc_view* b, const char* b_labels, float beta, const lc_view* c,
                             const char* c_labels) {
  return contract_impl(ctx, stream, alpha, a, a_labels, b, b_labels, beta, c, c_labels, nullptr, false);
}

lc_status lc_contract(lc_context* ctx, float alpha, const lc_view* a, const char* a_labels, const lc_view* b,
                      const char* b_labels, float beta, const lc_view* c, const char* c_labels) {
  lc_status st = lc_encode_contract(ctx, nullptr, alpha, a, a_labels, b, b_labels, beta, c, c_labels);
  return st ? st : lc_sync(ctx, nullptr);
}

lc_status lc_plan_contract(lc_context* ctx, float alpha, const lc_view* a, const char* a_labels, const lc_view* b,
                           const char* b_labels, float beta, const lc_view* c, const char* c_labels,
                           lc_contract_plan* out) {
  if (out == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null plan output");
  return contract_impl(ctx, nullptr, alpha, a, a_labels, b, b_labels, beta, c, c_labels, out, true);
}

lc_status lc_encode_gemm(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b, float beta,
                         const lc_view* c) {
  return gemm_impl(ctx, stream, alpha, a, b, beta, c, true);
}

lc_status lc_encode_gemm_fused(lc_context* ctx, void* stream, float alpha, const lc_view* a, const lc_view* b,
                               float beta, const lc_view* c, const lc_epilogue* epi) {
  return gemm_fused_impl(ctx, stream, alpha, a, b, beta, c, epi);
}

lc_status lc_gemm(lc_context* ctx, float alpha, const lc_view* a, const lc_view* b, float beta, const lc_view* c) {
  lc_status st = lc_encode_gemm(ctx, nullptr, alpha, a, b, beta, c);
  return st ? st : lc_sync(ctx, nullptr);
}

// crates/core/src/lib.rs:143-164 and crates/cpu/src/lib.rs:203-295: checks in the contract's
// order (Shape, Dtype, Alias, UnsupportedLayout, buffer range), then the tensor-core GEMM.
lc_status lc_backend_gemm(lc_context* ctx, void* stream, const lc_view* a, const lc_view* b, const lc_view* c,
                          float alpha, float beta) {
  if (ctx == nullptr || a == nullptr || b == nullptr || c == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (a->rank != 2 || b->rank != 2 || c->rank != 2) return fail(LC_ERR_SHAPE, "gemm operands are matrices");
  const uint64_t m = a->shape[0], k = a->shape[1], n = b->shape[1];
  if (b->shape[0] != k || c->shape[0] != m || c->shape[1] != n) return fail(LC_ERR_SHAPE, "gemm extents disagree");
  if (a->dtype != b->dtype || a->dtype != c->dtype) return fail(LC_ERR_DTYPE, "gemm dtypes differ");
  if (a->dtype != LC_F32 && a->dtype != LC_F16 && a->dtype != LC_BF16) return fail(LC_ERR_DTYPE, "gemm dtype");
  if (a->data == b->data || a->data == c->data || b->data == c->data) return fail(LC_ERR_ALIAS, "gemm operands share storage");
  auto layout = [](const lc_view& t) -> int {  // 0 row-major, 1 transposed, -1 other
    if (t.offset != 0) return -1;
    if (t.strides[1] == 1 && t.strides[0] == t.shape[1]) return 0;
    if (t.strides[0] == 1 && t.strides[1] == t.shape[0]) return 1;
    return -1;
  };
  const int la = layout(*a), lb = layout(*b), lcv = layout(*c);
  const bool ok = lcv == 0 && ((la == 0 && lb == 0) || (la == 1 && lb == 0) || (la == 0 && lb == 1));
  if (!ok) return fail(LC_ERR_UNSUPPORTED_LAYOUT, "gemm layout is not one of the three supported");
  const size_t es = dtype_size(a->dtype);
  auto range_ok = [&](const lc_view& t) {
    uint64_t last;
    if (is_empty(t)) return true;
    if (!max_index(t, &last)) return false;
    return (last + 1) * es <= t.buffer_bytes;
  };
  if (m > 0 && n > 0) {
    if (!range_ok(*c)) return fail(LC_ERR_SHAPE, "C buffer too short");
    if (alpha != 0.0f && k > 0 && (!range_ok(*a) || !range_ok(*b))) return fail(LC_ERR_SHAPE, "operand buffer too short");
  }
  return gemm_impl(ctx, stream, alpha, a, b, beta, c, false);
}

}  // extern "C"
