"""Oracle parity of the exact kernels and shapes the benchmark times, through the C ABI.

Every product here is compared with the CPU backend's sequential f32 product
(crates/cpu/src/lib.rs:664-691, restated in oracle/linalg_oracle.c), in full where the oracle
finishes in seconds and on sampled entries where it does not (as tests/contraction_test.rs:
1204-1227 samples the large products).  Tolerance: normwise max|C - C_cpu| / max|C_cpu| <= 1e-2
for bf16 inputs, <= 1e-5 (plus the CPU's own distance from the exact sum) for f32.  Each test
also asserts which kernel ran, so a planner change cannot move the benchmark onto an untested
kernel.  Complex argmax is checked against `ref_argmax_complex` (tests/argmax_test.rs:74-76).
"""
import os

import numpy as np
import pytest
import torch

import linalg_b200 as lb
from linalg_b200 import data
from oracle import oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
F32_TOL = 1e-5
D = 8192
THREADS = max(1, min(32, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def ctx(gpu):
    return lb.Context(0)


@pytest.fixture(scope="module")
def weights(gpu):
    """One bf16 weight matrix of the pipeline's layers: N(0, 1/8192), [in = 8192, out = 8192]."""
    w = torch.from_numpy(data.normal(31, (D, D), scale=D ** -0.5)).cuda().bfloat16()
    return w, u16(w)


def u16(t: torch.Tensor) -> np.ndarray:
    """Raw bits of a 16-bit tensor, as the oracle reads them."""
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def f32_of(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def bf16_dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


def normwise(got, want) -> float:
    want = np.asarray(want, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - want).max() / max(np.abs(want).max(), 1e-30))


def launched(ctx, name: str, last: int = 4) -> bool:
    return name in ctx.debug_launches()[-last:]


def oracle_product(a_bits, b_bits, m, n, k, b_strides=None) -> np.ndarray:
    out = np.zeros((m, n), np.float32)
    O.gemm3(O.DT_BF16, O.DT_BF16, O.DT_F32, a_bits, b_bits, out, 1.0, 0.0, b_strides=b_strides,
            threads=THREADS, shape=(m, n, k))
    return out


# ------------------------------------------------------------------------------------------------
# the square product (the contraction figure): 8192^3 bf16 on 256 x 256 tiles over CTA pairs
# ------------------------------------------------------------------------------------------------

def test_square_bf16_8192_on_two_sm_tiles_sampled(ctx):
    a = bf16_dev(data.uniform(40, (D, D)))
    b = bf16_dev(data.uniform(41, (D, D)))
    c = torch.empty(D, D, device="cuda", dtype=torch.bfloat16)
    lb.encode_gemm(ctx, None, 1.0, a, b, 0.0, c)
    ctx.sync()
    assert launched(ctx, "gemm_bf16_2sm_n256", 1), ctx.debug_launches()[-4:]
    rng = np.random.default_rng(40)
    rows, cols = rng.integers(0, D, 512), rng.integers(0, D, 512)
    cpu = O.gemm_entries(O.DT_BF16, u16(a), u16(b), D, rows, cols, n=D)
    got = f32_of(c[torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()])
    assert normwise(got, cpu) <= BF16_TOL


# ------------------------------------------------------------------------------------------------
# the pipeline's products at the benchmark width, with their fused epilogues
# ------------------------------------------------------------------------------------------------

@pytest.mark.parametrize("kind", ["generic", "relu"])
def test_forward_product_on_cta_pairs_full(ctx, weights, kind):
    """H[l+1] = relu(H[l] @ W): [64, 8192] x [8192, 8192], computed as C^T = W^T H^T on 64-wide
    tiles with K split over a CTA pair, the product every stage of a multi-GPU run streams."""
    w, wbits = weights
    x = bf16_dev(data.normal(42, (64, D)))
    y = torch.empty(64, D, device="cuda", dtype=torch.bfloat16)
    epi = lb.EPI_RELU if kind == "relu" else lb.EPI_NONE
    lb.encode_gemm_fused(ctx, None, 1.0, x, w, 0.0, y, epi)
    ctx.sync()
    assert launched(ctx, "gemm_bf16_pair_n64", 1), ctx.debug_launches()[-4:]
    cpu = oracle_product(u16(x), wbits, 64, D, D)
    want = np.maximum(cpu, 0.0) if kind == "relu" else cpu
    got = f32_of(y)
    assert normwise(got, want) <= BF16_TOL
    if kind == "relu":
        # clearly negative pre-activations (beyond any rounding) come out as zero
        assert (got[cpu < -BF16_TOL * np.abs(cpu).max()] == 0).all()
        assert (got >= 0).all()


def test_data_gradient_on_cta_pairs_with_relu_mask_full(ctx, weights):
    """dP[l-1] = (dP[l] @ W^T) where H[l] > 0: the ReLU derivative fused into the data gradient."""
    w, wbits = weights
    dp = bf16_dev(data.normal(43, (64, D), scale=1e-3))
    h = bf16_dev(data.normal(44, (64, D)))
    out = torch.empty(64, D, device="cuda", dtype=torch.bfloat16)
    lb.encode_gemm_fused(ctx, None, 1.0, dp, w.t(), 0.0, out, lb.EPI_RELU_MASK, aux=h)
    ctx.sync()
    assert launched(ctx, "gemm_bf16_pair_n64", 1), ctx.debug_launches()[-4:]
    cpu = oracle_product(u16(dp), wbits, 64, D, D, b_strides=(1, D))
    keep = f32_of(h) > 0
    want = np.where(keep, cpu, 0.0)
    got = f32_of(out)
    assert normwise(got, want) <= BF16_TOL
    assert (got[~keep] == 0).all() and not np.signbit(got[~keep]).any()  # +0 where the mask is off


@pytest.mark.parametrize("which", ["forward", "data_gradient"])
def test_grouped_product_as_the_one_stage_step_plans_it(ctx, weights, which):
    """A stage holding every layer runs four microbatches as one [256, 8192] x [8192, 8192]
    product, pinned to the one-microbatch product's split (2) and orientation (C^T = W^T H^T) on a
    256-wide tile, so each weight tile is read once for the whole group.  It must equal the four
    one-microbatch products bit for bit (and the same product on 128 x 256 CTA-pair tiles,
    LC_GEMM_QUAD=0, which the pipeline grouping test compares) and the oracle within tolerance."""
    w, wbits = weights
    fwd = which == "forward"
    rows = 256
    a = bf16_dev(data.normal(45, (rows, D), scale=1.0 if fwd else 1e-3))
    h = bf16_dev(data.normal(46, (rows, D)))
    b = w if fwd else w.t()
    epi = lb.EPI_RELU if fwd else lb.EPI_RELU_MASK
    grouped = torch.empty(rows, D, device="cuda", dtype=torch.bfloat16)
    lb.encode_gemm_fused(ctx, None, 1.0, a, b, 0.0, grouped, epi, aux=None if fwd else h, tile_n=256, splits=2,
                         swap=1)
    ctx.sync()
    # 256 x 256 tiles on clusters of 4 (two CTA pairs with cta_group::2 MMAs, one per K half)
    assert launched(ctx, "gemm_bf16_quad_n256", 1), ctx.debug_launches()[-4:]
    single = torch.empty_like(grouped)
    for j in range(4):
        sl = slice(64 * j, 64 * j + 64)
        lb.encode_gemm_fused(ctx, None, 1.0, a[sl], b, 0.0, single[sl], epi, aux=None if fwd else h[sl])
    ctx.sync()
    assert torch.equal(grouped.view(torch.int16), single.view(torch.int16))
    cpu = oracle_product(u16(a), wbits, rows, D, D, b_strides=None if fwd else (1, D))
    want = np.maximum(cpu, 0.0) if fwd else np.where(f32_of(h) > 0, cpu, 0.0)
    assert normwise(f32_of(grouped), want) <= BF16_TOL


def test_weight_gradient_with_fused_sgd_on_two_sm_tiles_sampled(ctx):
    """W -= lr * H^T @ dP over the whole batch (K = 2048), bf16 copy written beside the f32
    master: the step's weight update at the benchmark width, on 256 x 256 tiles over CTA pairs."""
    B, lr = 2048, 1e-3
    hb = bf16_dev(data.normal(47, (B, D)))
    dpb = bf16_dev(data.normal(48, (B, D), scale=1e-3))
    master = torch.from_numpy(data.normal(49, (D, D), scale=D ** -0.5)).cuda()
    m0 = master.cpu().numpy()
    wb = torch.empty(D, D, device="cuda", dtype=torch.bfloat16)
    lb.encode_gemm_fused(ctx, None, 1.0, hb.t(), dpb, 1.0, master, lb.EPI_SGD, aux2=wb, lr=lr)
    ctx.sync()
    assert launched(ctx, "gemm_bf16_2sm_n256", 1), ctx.debug_launches()[-4:]
    rng = np.random.default_rng(47)
    rows, cols = rng.integers(0, D, 512), rng.integers(0, D, 512)
    g = O.gemm_entries(O.DT_BF16, u16(hb), u16(dpb), B, rows, cols, a_strides=(1, D), b_strides=(D, 1))
    update = (np.float32(lr) * g).astype(np.float32)
    want = (m0[rows, cols] - update).astype(np.float32)
    got = master.cpu().numpy()
    assert np.abs(got[rows, cols].astype(np.float64) - want).max() <= BF16_TOL * np.abs(update).max()
    # the compute copy is the nearest-even bf16 of the updated master (crates/cpu/src/lib.rs:725-731)
    assert np.array_equal(O.f32_to_bf16(got), u16(wb))


# ------------------------------------------------------------------------------------------------
# the tall split-K configs: M = N = 256, K = 262144, inputs N(0, 1) / sqrt(K), seeds 0 and 1
# ------------------------------------------------------------------------------------------------

@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_tall_split_k_config_against_the_sequential_product(ctx, dtype):
    """Against the CPU backend's k-order product (not a GPU f64 matmul), on a 32 x 64 grid of
    entries.  The CPU's own f32 sum over 262144 terms drifts from the exact value by about
    sqrt(K) ulp, so the GPU must sit within the tolerance of the exact (f64) sum and within the
    tolerance plus the CPU's own error of the CPU's result."""
    K = 262144
    a = data.normal(0, (256, K), scale=K ** -0.5)
    b = data.normal(1, (K, 256), scale=K ** -0.5)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    if dtype == "bf16":
        ta, tb = ta.bfloat16(), tb.bfloat16()
    tc = torch.zeros(256, 256, device="cuda", dtype=ta.dtype)
    lb.contract(ctx, 1.0, (ta, "ik"), (tb, "kj"), 0.0, (tc, "ij"))
    plan = lb.plan_contract(ctx, 1.0, (ta, "ik"), (tb, "kj"), 0.0, (tc, "ij"))
    assert plan["kind"] == "Split" and plan["splits"] > 2, plan
    rng = np.random.default_rng(262144)
    rows = np.sort(rng.choice(256, 32, replace=False))
    cols = np.sort(rng.choice(256, 64, replace=False))
    rr, cc = (g.ravel() for g in np.meshgrid(rows, cols, indexing="ij"))
    if dtype == "f32":
        an, bn = a, b
        cpu = O.gemm_entries(O.DT_F32, a, b, K, rr, cc, n=256)
    else:
        an, bn = f32_of(ta), f32_of(tb)
        cpu = O.gemm_entries(O.DT_BF16, u16(ta), u16(tb), K, rr, cc, n=256)
    exact = (an[rows].astype(np.float64) @ bn[:, cols].astype(np.float64)).ravel()
    got = f32_of(tc)[rr, cc].astype(np.float64)
    tol = F32_TOL if dtype == "f32" else BF16_TOL
    denom = np.abs(exact).max()
    cpu_err = np.abs(cpu - exact).max() / denom
    assert np.abs(got - exact).max() / denom <= tol
    assert np.abs(got - cpu).max() / denom <= tol + cpu_err


# ------------------------------------------------------------------------------------------------
# complex argmax (src/ops/argmax.rs:106-131, shaders/argmax.metal:162-203)
# ------------------------------------------------------------------------------------------------

def gpu_argmax_complex(ctx, z: np.ndarray, kind: int, stride: int = 1, n: int | None = None) -> int:
    """z: complex64 values; the view takes n of them at `stride` complex elements."""
    t = torch.from_numpy(np.ascontiguousarray(z).astype(np.complex64)).cuda()
    n = t.numel() if n is None else n
    v = lb.View.raw(t, 0, [n], [stride])
    out = torch.full((1,), 0xDEADBEEF, dtype=torch.uint32, device="cuda")
    lb.argmax_complex(ctx, v, "L1" if kind == O.MAG_L1 else "Hypot", out)
    return int(out.cpu().numpy()[0])


def as_complex(pairs: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(pairs, dtype=np.float32).view(np.complex64).reshape(-1)


def test_argmax_complex_reference_known_answers(ctx):
    import json
    from pathlib import Path
    G = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())
    bits = lambda h: np.array([int(h, 16)], np.uint32).view(np.float32)[0]
    for case in G["argmax_complex"]["cases"]:
        z = np.empty((case["n"], 2), np.float32)
        z[:] = (bits(case["fill"][0]), bits(case["fill"][1]))
        for i, re, im in case["set"]:
            z[i] = (bits(re), bits(im))
        for kind, want in case["expected"].items():
            k = O.MAG_L1 if kind == "l1" else O.MAG_HYPOT
            assert gpu_argmax_complex(ctx, as_complex(z), k) == want, (case["cite"], kind)


@pytest.mark.parametrize("kind", [0, 1])
def test_argmax_complex_random_sizes_and_strides(ctx, kind):
    """Random values over the single-pass / two-pass boundaries (4096 and 1024 x groups) and
    strided rows and columns of a matrix with an offset (tests/argmax_test.rs:413-441, :488-507)."""
    for n in (1, 2, 255, 256, 257, 4095, 4096, 4097, 262145, 1_000_003):
        z = as_complex(data.uniform(500 + n, (n, 2)) * np.float32(50))
        assert gpu_argmax_complex(ctx, z, kind) == O.argmax_complex(z, kind), n
    z = as_complex(data.uniform(77, (10_000_000, 2)))
    assert gpu_argmax_complex(ctx, z, kind) == O.argmax_complex(z, kind)
    m = as_complex(data.uniform(18, (1000 * 1000, 2)) * np.float32(50)).reshape(1000, 1000)
    for line in (0, 1, 499, 998, 999):
        col = np.ascontiguousarray(m[:, line])
        t = torch.from_numpy(m).cuda()
        v = lb.View.raw(t, line, [1000], [1000])
        out = torch.zeros(1, dtype=torch.uint32, device="cuda")
        lb.argmax_complex(ctx, v, "L1" if kind == 0 else "Hypot", out)
        assert int(out.cpu().numpy()[0]) == O.argmax_complex(col, kind), line


def test_argmax_complex_ties_nans_and_extremes(ctx):
    m = np.finfo(np.float32).max
    for kind in (0, 1):
        for n in (1, 2, 3, 257, 4097, 100_003):
            ties = as_complex(np.tile(np.float32([3.0, -4.0]), (n, 1)))
            assert gpu_argmax_complex(ctx, ties, kind) == 0
            if n >= 3:
                x = np.tile(np.float32([1.0, 1.0]), (n, 1))
                x[n // 3] = (np.inf, 0.0)
                for p in (0, n // 2, n - 1):
                    y = x.copy()
                    y[p] = (np.nan, 1.0) if p % 2 == 0 else (np.inf, np.nan)
                    zz = as_complex(y)
                    assert gpu_argmax_complex(ctx, zz, kind) == O.argmax_complex(zz, kind) == p
        big = np.tile(np.float32([0.6, 0.6]) * m, (5000, 1))
        big[4999] = np.float32([0.9, 0.3]) * m
        zb = as_complex(big)
        assert gpu_argmax_complex(ctx, zb, kind) == O.argmax_complex(zb, kind)


# ------------------------------------------------------------------------------------------------
# fused GELU epilogues (f32, the reference-mode pipeline's layers)
# ------------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,n,k", [(64, 512, 768), (200, 96, 130_001), (33, 1000, 64)])
def test_gelu_epilogues_equal_the_unfused_sequence(ctx, m, n, k):
    """gemm -> gelu and gemm -> gelu_backward (crates/pipeline/src/lib.rs:176-178, :211-220) as
    one product each: bit-identical to lc_encode_gemm followed by the standalone lc_gelu /
    lc_gelu_backward, and within tolerance of the oracle's gemm + gelu.  The long-K case splits."""
    x = torch.from_numpy(data.uniform(60 + k, (m, k))).cuda()
    w = torch.from_numpy(data.uniform(61 + k, (k, n)) * np.float32(k ** -0.5)).cuda()
    pre_ref = torch.empty(m, n, device="cuda")
    lb.encode_gemm(ctx, None, 1.0, x, w, 0.0, pre_ref)
    act_ref = torch.empty_like(pre_ref)
    lb.gelu(ctx, pre_ref, act_ref)
    act = torch.empty_like(pre_ref)
    pre = torch.empty_like(pre_ref)
    lb.encode_gemm_fused(ctx, None, 1.0, x, w, 0.0, act, lb.EPI_GELU, aux2=pre)
    ctx.sync()
    assert torch.equal(pre.view(torch.int32), pre_ref.view(torch.int32))
    assert torch.equal(act.view(torch.int32), act_ref.view(torch.int32))
    cpu = np.zeros((m, n), np.float32)
    O.gemm3(O.DT_F32, O.DT_F32, O.DT_F32, x.cpu().numpy(), w.cpu().numpy(), cpu, 1.0, 0.0, threads=THREADS)
    assert normwise(act.cpu().numpy(), O.gelu(cpu)) <= 1e-4
    # backward: dpre = gelu'(pre) * (g @ W^T), g the gradient arriving at the layer's output
    g = torch.from_numpy(data.uniform(62 + k, (m, n))).cuda()
    dx_ref = torch.empty(m, k, device="cuda")
    pre_in = torch.from_numpy(data.normal(63 + k, (m, k))).cuda()  # the layer below's pre-activation
    lb.encode_gemm(ctx, None, 1.0, g, w.t(), 0.0, dx_ref)
    dpre_ref = torch.empty_like(dx_ref)
    lb.gelu_backward(ctx, pre_in, dx_ref, dpre_ref)
    dpre = torch.empty_like(dx_ref)
    lb.encode_gemm_fused(ctx, None, 1.0, g, w.t(), 0.0, dpre, lb.EPI_GELU_BACKWARD, aux=pre_in)
    ctx.sync()
    assert torch.equal(dpre.view(torch.int32), dpre_ref.view(torch.int32))


def test_fused_epilogue_argument_checks(ctx):
    a = torch.zeros(64, 64, device="cuda")
    b = torch.zeros(64, 64, device="cuda")
    c = torch.zeros(64, 64, device="cuda")
    with pytest.raises(lb.DtypeError):
        lb.encode_gemm_fused(ctx, None, 1.0, a, b, 0.0, c, lb.EPI_RELU_MASK, aux=c)  # f32 inputs
    with pytest.raises(lb.InvalidArgument):
        lb.encode_gemm_fused(ctx, None, 1.0, a, b, 0.0, c, lb.EPI_GELU_BACKWARD)  # no pre-activation
    with pytest.raises(lb.ShapeError):
        lb.encode_gemm_fused(ctx, None, 1.0, a, b, 0.0, c, lb.EPI_GELU_BACKWARD, aux=torch.zeros(64, 32, device="cuda"))
    with pytest.raises(lb.InvalidArgument):
        lb.encode_gemm_fused(ctx, None, 1.0, a, b, 0.0, c, 9)
    ab, bb = a.bfloat16(), b.bfloat16()
    with pytest.raises(lb.DtypeError):
        lb.encode_gemm_fused(ctx, None, 1.0, ab, bb, 0.0, c.bfloat16(), lb.EPI_GELU)
