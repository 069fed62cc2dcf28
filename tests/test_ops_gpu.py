"""GPU parity of the op API against the CPU oracle, through the C ABI.

Bit-exact for permute / slice-pack / argmax indices / sqrt / reciprocal; contraction within the
reference's componentwise f64 gate (tests/contraction_test.rs:1-13) and normwise
max|C - C_cpu| / max|C_cpu| <= 1e-5 (f32, 3xTF32) or 1e-2 (bf16) against the CPU backend's
sequential f32 product.
"""
import itertools

import numpy as np
import pytest
import torch

import linalg_b200 as lb
from linalg_b200 import data
from oracle import oracle as O

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_TOL = 1e-2


@pytest.fixture(scope="module")
def ctx(gpu):
    return lb.Context(0)


def dev(x: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def bits(t) -> np.ndarray:
    a = t.detach().cpu().contiguous()
    if a.dtype == torch.float32:
        return a.view(torch.int32).numpy().view(np.uint32)
    return a.numpy()


SPECIALS = np.array([0x00000000, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x7F800001,
                     0x7FFFFFFF, 0xBF800000, 0xFF7FFFFF, 0x80000001, 0x807FFFFF, 0x00000001, 0x007FFFFF,
                     0x00800000, 0x3F800000, 0x40000000, 0x7F7FFFFF, 0x3F000000, 0x00200001, 0x7E800000,
                     0x7F000000, 0x00400000, 0x7F2AAAAA], dtype=np.uint32)


def same_bits_or_both_nan(got: np.ndarray, want: np.ndarray):
    g = got.view(np.float32)
    w = want.view(np.float32)
    ok = (got == want) | (np.isnan(g) & np.isnan(w))
    assert ok.all(), np.nonzero(~ok)[0][:10]


# ------------------------------------------------------------------------------------------------
# sqrt / reciprocal
# ------------------------------------------------------------------------------------------------

@pytest.mark.parametrize("op", ["sqrt", "reciprocal"])
def test_elementwise_specials_and_binades(ctx, op):
    rng = np.random.default_rng(5)
    # every binade, both signs, plus the specials
    fields = np.arange(0, 256, dtype=np.uint32)
    mant = rng.integers(0, 1 << 23, size=(256, 64), dtype=np.uint32)
    xs = ((fields[:, None] << 23) | mant).ravel()
    xs = np.concatenate([SPECIALS, xs, xs | 0x80000000]).view(np.float32)
    src = dev(xs)
    dst = torch.empty_like(src)
    getattr(lb, op)(ctx, src, dst)
    want = O.sqrt(xs) if op == "sqrt" else O.reciprocal(xs)
    same_bits_or_both_nan(bits(dst), want.view(np.uint32))
    if op == "reciprocal":
        # NaN payload and sign survive, quietened
        nan_in = xs.view(np.uint32)
        isn = np.isnan(xs)
        assert (bits(dst)[isn] == (nan_in[isn] | 0x00400000)).all()


@pytest.mark.parametrize("op", ["sqrt", "reciprocal"])
def test_elementwise_strided_inplace_and_tail(ctx, op):
    x = np.abs(data.normal(3, (37, 53))) + np.float32(1e-3)
    base = dev(np.zeros(4000, np.float32))
    base[5:5 + 37 * 53] = dev(x.ravel())
    view = lb.View.raw(base, 5, [37, 53], [53, 1])
    # strided: every other column into a separate buffer
    dst = dev(np.zeros((37, 27), np.float32))
    sv = lb.View.raw(base, 5, [37, 27], [53, 2])
    getattr(lb, op)(ctx, sv, dst)
    f = O.sqrt if op == "sqrt" else O.reciprocal
    assert (bits(dst) == f(x[:, ::2]).view(np.uint32)).all()
    # in place over the misaligned (offset 5) contiguous view
    getattr(lb, op)(ctx, view, view)
    assert (bits(base[5:5 + 37 * 53]) == f(x).ravel().view(np.uint32)).all()
    # overlap that is not the same view is rejected
    other = lb.View.raw(base, 6, [37, 53], [53, 1])
    with pytest.raises(lb.Overlap):
        getattr(lb, op)(ctx, view, other)


@pytest.mark.parametrize("op", ["sqrt", "reciprocal"])
def test_elementwise_baseline_tensor_bit_exact(ctx, op):
    x = np.abs(data.normal(0, (64, 128, 128, 64))) + np.float32(1e-3)
    src = dev(x)
    dst = torch.empty_like(src)
    getattr(lb, op)(ctx, src, dst)
    want = O.sqrt(x) if op == "sqrt" else O.reciprocal(x)
    assert (bits(dst) == want.view(np.uint32)).all()


# ------------------------------------------------------------------------------------------------
# complex reciprocal (src/ops/reciprocal.rs:17-31)
# ------------------------------------------------------------------------------------------------

def gpu_rcp_c32(ctx, z: np.ndarray) -> np.ndarray:
    src = dev(np.ascontiguousarray(z, dtype=np.complex64))
    dst = torch.empty_like(src)
    lb.reciprocal(ctx, src, dst)
    return dst.cpu().numpy()


def test_complex_reciprocal_goldens(ctx):
    """Every exact complex result the reference's tests assert (tests/reciprocal_test.rs:569-741),
    bit for bit, and the NaN rule."""
    from test_oracle_golden import G, c32_of
    g = G["reciprocal_c32"]
    zs = np.array([c32_of(e["z"]) for e in g["exact"]], np.complex64)
    got = gpu_rcp_c32(ctx, zs).view(np.uint32).reshape(-1, 2)
    want = np.array([[int(e["w"][0], 16), int(e["w"][1], 16)] for e in g["exact"]], np.uint32)
    assert (got == want).all(), np.argwhere(got != want)[:5]
    nz = np.array([c32_of(p) for p in g["nan_inputs"]], np.complex64)
    assert (gpu_rcp_c32(ctx, nz).view(np.uint32) == 0x7FC00000).all()


@pytest.mark.parametrize("seed,lo,hi,spread", [(10, 87, 167, 80), (11, 87, 167, 2), (12, -22, 254, 276),
                                               (20, 245, 254, 9), (30, -22, 3, 25), (31, -22, 60, 82)])
def test_complex_reciprocal_bit_exact_and_gate(ctx, seed, lo, hi, spread):
    """300,000 inputs per family (moderate, comparable parts, full range, near overflow, near
    underflow): bit for bit the oracle's split-float Smith algorithm, and within the reference's
    accuracy gate against the f64 value."""
    from test_oracle_golden import complex_inputs, assert_complex_gate
    z = complex_inputs(seed + 100, 300_000, lo, hi, spread)
    got = gpu_rcp_c32(ctx, z)
    want = O.reciprocal_c32(z)
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    assert_complex_gate(z, got)


def test_complex_reciprocal_specials_and_real_axis(ctx):
    """Zero, infinite and NaN parts in every sign combination, and 1/(x + 0i) on the real axis
    equal to the real reciprocal with imaginary part -0 (tests/reciprocal_test.rs:745-760)."""
    specials = SPECIALS.view(np.float32)
    re, im = np.meshgrid(specials, specials)
    z = np.empty(re.size, np.complex64)
    z.real, z.imag = re.ravel(), im.ravel()
    got = gpu_rcp_c32(ctx, z)
    assert (got.view(np.uint32) == O.reciprocal_c32(z).view(np.uint32)).all()
    from test_oracle_golden import fields_to_f32
    x = fields_to_f32(np.random.default_rng(40), np.random.default_rng(41).integers(-22, 255, 100_000))
    w = gpu_rcp_c32(ctx, x.astype(np.complex64))
    assert (w.real.view(np.uint32) == O.reciprocal(x).view(np.uint32)).all()
    assert (w.imag.view(np.uint32) == 0x80000000).all()


def test_complex_reciprocal_layouts(ctx):
    """Strided (every other element), a misaligned start and an odd count (no 16-byte vectors),
    in place, and a batched diagonal view: each element gets its own reciprocal."""
    from test_oracle_golden import complex_inputs
    z = complex_inputs(50, 4001, 100, 150, 10)
    base = dev(z)
    want = O.reciprocal_c32(z)
    # every other element into a dense buffer
    sv = lb.View.raw(base, 0, [2001], [2])
    out = torch.zeros(2001, dtype=torch.complex64, device="cuda")
    lb.reciprocal(ctx, sv, out)
    assert (out.cpu().numpy().view(np.uint32) == np.ascontiguousarray(want[::2]).view(np.uint32)).all()
    # misaligned start (offset 1: 8-byte aligned only), odd count, out of place
    mv = lb.View.raw(base, 1, [3999], [1])
    out2 = torch.zeros(3999, dtype=torch.complex64, device="cuda")
    lb.reciprocal(ctx, mv, out2)
    assert (out2.cpu().numpy().view(np.uint32) == want[1:4000].view(np.uint32)).all()
    # the diagonals of a batch of 7 x 7 matrices, in place
    m = complex_inputs(51, 5 * 49, 100, 150, 10)
    mt = dev(m)
    diag = lb.View.raw(mt, 0, [5, 7], [49, 8])
    lb.reciprocal(ctx, diag, diag)
    got = mt.cpu().numpy().reshape(5, 7, 7)
    ref = m.reshape(5, 7, 7).copy()
    idx = np.arange(7)
    ref[:, idx, idx] = O.reciprocal_c32(ref[:, idx, idx].ravel()).reshape(5, 7)
    assert (got.view(np.uint32) == ref.view(np.uint32)).all()


# ------------------------------------------------------------------------------------------------
# permutation
# ------------------------------------------------------------------------------------------------

def check_permute(ctx, x: np.ndarray, perm, dtype=None):
    t = dev(x)
    pv = lb.permute_view(lb.View.of(t, dtype), perm)
    out = torch.empty(pv.shape, dtype=t.dtype, device="cuda")
    lb.materialize(ctx, pv, out)
    want = O.gather(x.view(np.uint32) if x.dtype == np.float32 else x, pv.offset, pv.shape, pv.strides)
    got = bits(out) if x.dtype == np.float32 else out.cpu().numpy()
    assert (got == want).all()


@pytest.mark.parametrize("rank", [1, 2, 3, 4, 5])
def test_permute_all_permutations_prime_extents(ctx, rank):
    primes = [3, 5, 7, 11, 13][:rank]
    x = data.uniform(rank, primes)
    for perm in itertools.permutations(range(rank)):
        check_permute(ctx, x, list(perm))


def test_permute_tiles_edges_and_complex(ctx):
    x = data.uniform(9, (70, 130))
    check_permute(ctx, x, [1, 0])
    x = data.uniform(10, (3, 65, 129, 2))
    check_permute(ctx, x, [0, 2, 1, 3])
    check_permute(ctx, x, [3, 1, 2, 0])
    # complex (8-byte) transpose and the conjugate flag
    z = (data.normal(11, (33, 47)) + 1j * data.normal(12, (33, 47))).astype(np.complex64)
    t = dev(z)
    out = torch.empty((47, 33), dtype=torch.complex64, device="cuda")
    lb.adjoint(ctx, t, out)
    assert (out.cpu().numpy() == np.conj(z.T)).all()
    lb.adjoint(ctx, out, t2 := torch.empty_like(t))
    assert (t2.cpu().numpy().view(np.uint64) == z.view(np.uint64)).all()  # involution, bitwise


def test_permute_baseline_bit_exact(ctx):
    x = data.normal(0, (64, 128, 128, 64))
    check_permute(ctx, x, [0, 3, 1, 2])


# ------------------------------------------------------------------------------------------------
# slicing / pack / concat
# ------------------------------------------------------------------------------------------------

def test_slice_pack_baseline_bit_exact(ctx):
    x = data.normal(0, (64, 128, 128, 64))
    t = dev(x)
    s = lb.slice(t, [range(0, 64), range(32, 96), range(0, 128), range(16, 48)])
    out = torch.empty(s.shape, dtype=torch.float32, device="cuda")
    lb.pack(ctx, s, out)
    assert (bits(out) == np.ascontiguousarray(x[:, 32:96, :, 16:48]).view(np.uint32)).all()


@pytest.mark.parametrize("dtype,npdt", [(torch.float16, np.float16), (torch.float32, np.float32),
                                        (torch.float64, np.float64), (torch.complex128, np.complex128)])
def test_pack_misaligned_rows_all_element_sizes(ctx, dtype, npdt):
    rng = np.random.default_rng(21)
    raw = rng.integers(0, 255, size=(9 * 23 * npdt().itemsize + 64), dtype=np.uint8)
    n = (raw.size - 64) // npdt().itemsize
    x = raw[: n * npdt().itemsize].view(npdt).reshape(9, 23)
    t = dev(x)
    for r0, c0 in ((0, 0), (1, 1), (2, 3), (0, 5)):
        s = lb.slice(t, [range(r0, 9), range(c0, 23)])
        dst_base = torch.zeros(400, dtype=dtype, device="cuda")
        dst = lb.View.raw(dst_base, 3, s.shape, [s.shape[1] + 2, 1])
        lb.pack(ctx, s, dst)
        got = dst_base.cpu().numpy()
        want = x[r0:, c0:]
        for i in range(want.shape[0]):
            row = got[3 + i * (s.shape[1] + 2): 3 + i * (s.shape[1] + 2) + s.shape[1]]
            assert (row.view(np.uint8) == np.ascontiguousarray(want[i]).view(np.uint8)).all()


def test_concat(ctx):
    parts = [data.uniform(i, (4, w, 3)) for i, w in enumerate([2, 0, 5, 1])]
    out = torch.empty((4, 8, 3), dtype=torch.float32, device="cuda")
    lb.concat(ctx, [dev(p) for p in parts], 1, out)
    assert (bits(out) == np.concatenate(parts, axis=1).view(np.uint32)).all()


# ------------------------------------------------------------------------------------------------
# argmax
# ------------------------------------------------------------------------------------------------

def gpu_argmax(ctx, x: np.ndarray) -> int:
    t = dev(x.astype(np.float32))
    out = torch.full((1,), 0xDEADBEEF, dtype=torch.uint32, device="cuda")
    lb.argmax(ctx, t, out)
    return int(out.cpu().numpy()[0])


def test_argmax_rank1_cases(ctx):
    for n in (1, 2, 255, 256, 257, 4095, 4096, 4097, 262143, 262144, 262145, 1_000_003):
        x = data.normal(n, (n,))
        assert gpu_argmax(ctx, x) == O.argmax(x), n
        y = np.full(n, 7.0, np.float32)
        y[::2] = -7.0
        assert gpu_argmax(ctx, y) == 0
        if n >= 3:
            z = np.ones(n, np.float32)
            z[n // 3] = np.inf
            z[n - 1] = np.nan
            assert gpu_argmax(ctx, z) == n - 1
            z[n // 2] = -np.nan
            assert gpu_argmax(ctx, z) == min(n // 2, n - 1)
    x = data.normal(14, (10_000_000,)) / np.float32(1000)
    x[-1] = 10.0
    x[5_000_000] = -10.0
    x[777] = -10.0
    assert gpu_argmax(ctx, x) == 777


def test_argmax_rows_baseline_bit_exact(ctx):
    x = data.normal(0, (64, 128, 128, 64))
    x[0, 0, 0, :] = 3.0          # tie storm: lowest index
    x[0, 0, 1, 10] = np.nan      # NaN wins
    x[0, 0, 2, 5] = -np.inf
    t = dev(x)
    out = torch.empty((64, 128, 128), dtype=torch.uint32, device="cuda")
    lb.argmax_rows(ctx, t, out)
    want = O.argmax_rows(x)
    assert (out.cpu().numpy() == want).all()
    assert want[0, 0, 0] == 0 and want[0, 0, 1] == 10 and want[0, 0, 2] == 5


def test_argmax_rows_strided_and_odd(ctx):
    x = data.normal(33, (17, 5, 45))
    t = dev(x)
    v = lb.permute_view(t, [0, 2, 1])  # rows along the length-5 axis, stride 45
    out = torch.empty((17, 45), dtype=torch.uint32, device="cuda")
    lb.argmax_rows(ctx, v, out)
    want = O.argmax_rows(np.ascontiguousarray(np.transpose(x, (0, 2, 1))))
    assert (out.cpu().numpy() == want).all()


@pytest.mark.parametrize("rows,cols,offset", [(7, 33, 0), (5, 64, 0), (3, 200, 0), (9, 1000, 0), (6, 96, 1)])
def test_argmax_rows_wide_and_misaligned(ctx, rows, cols, offset):
    """Rows wider than the 16 lanes that share one (several loads per lane), odd widths and a
    misaligned start (no 16-byte loads): ties across lanes, zero rows, NaN and infinities must
    give the reference's indices."""
    x = data.normal(rows * cols + offset, (rows, cols))
    x[0, :] = 0.0                                   # all zero: index 0
    if rows > 1:
        x[1, cols - 1] = 7.5
        x[1, 3] = -7.5                              # |x| tie across lanes: lowest index
    if rows > 2:
        x[2, cols // 2] = np.nan
        x[2, 1] = np.inf                            # NaN outranks inf
    if rows > 3:
        x[3, :] = np.nan                            # all NaN: index 0
    if rows > 4:
        x[4, cols - 2] = -np.inf
    flat = np.concatenate([np.zeros(offset, np.float32), x.ravel()])
    t = dev(flat)
    v = lb.View.raw(t, offset, [rows, cols], [cols, 1])
    out = torch.empty((rows,), dtype=torch.uint32, device="cuda")
    lb.argmax_rows(ctx, v, out)
    want = O.argmax_rows(x)
    assert (out.cpu().numpy() == want).all(), (out.cpu().numpy(), want)


@pytest.mark.parametrize("cols", [16, 32, 64, 128, 256, 512])
@pytest.mark.parametrize("rows", [1, 257, 3001])
def test_argmax_rows_power_of_two_widths(ctx, rows, cols):
    """The lane-scanning kernel for 16..512-float rows: each lane holds 16 values at columns
    4 * (lane + L * j) + e, so ties inside one lane, ties across lanes, NaN after and before an
    infinity, negative zero against zero, and a row count that leaves a partial pass must all
    give the reference's lowest-index-wins result."""
    x = data.normal(rows * 7 + cols, (rows, cols))
    specials = SPECIALS.view(np.float32)
    rng = np.random.default_rng(rows + cols)
    for r in range(0, rows, 3):              # rows with special values at random columns
        at = rng.choice(cols, size=min(6, cols), replace=False)
        x[r, at] = specials[rng.integers(0, len(specials), size=len(at))]
    x[0, :] = 0.0
    x[0, cols // 2] = -0.0                   # -0 ties +0: index 0
    if rows > 1:
        x[1, :] = 2.0
        x[1, 1] = -2.0                       # all tied: index 0
    if rows > 2:
        x[2, cols - 1] = np.nan
        x[2, 3] = np.inf                     # NaN outranks inf wherever it sits
    if rows > 3:
        x[3, 4 * (cols // 16) + 2] = 9.0     # one lane's second float4 against
        x[3, 2] = -9.0                       # the first lane's: the lower column wins
    if rows > 4:
        x[4, :] = np.nan                     # NaNs of several payloads after an infinity:
        x[4, 0] = -np.inf                    # the first NaN, index 1
        x[4, 1] = np.uint32(0x7fc00001).view(np.float32)
    t = dev(x)
    out = torch.empty((rows,), dtype=torch.uint32, device="cuda")
    lb.argmax_rows(ctx, t, out)
    want = O.argmax_rows(x)
    assert (out.cpu().numpy() == want).all(), np.nonzero(out.cpu().numpy() != want)[0][:10]


# ------------------------------------------------------------------------------------------------
# contraction
# ------------------------------------------------------------------------------------------------

def to_np_f32(t):
    return t.detach().float().cpu().numpy()


def gate_check(got64, a, al, b, bl, c0, cl, alpha, beta, cview_np=None):
    exact, mag, idx, k = O.contract_reference(alpha, a.ravel(), al, 0, a.shape, [s // a.itemsize for s in a.strides],
                                              b.ravel(), bl, 0, b.shape, [s // b.itemsize for s in b.strides],
                                              beta, c0.ravel(), cl, 0, c0.shape,
                                              [s // c0.itemsize for s in c0.strides])
    gate, _ = O.contraction_gate(got64.ravel()[idx.astype(np.int64)], exact, mag, k)
    return gate


def run_gemm_case(ctx, m, n, k, alpha=1.0, beta=0.0, dtype=torch.float32, seed=0, at=False, bt=False):
    a = data.uniform(seed, (m, k)) if not at else data.uniform(seed, (k, m)).T
    b = data.uniform(seed + 1, (k, n)) if not bt else data.uniform(seed + 1, (n, k)).T
    c0 = data.uniform(seed + 2, (m, n))
    ta = dev(np.ascontiguousarray(a.T)).T if at else dev(a)
    tb = dev(np.ascontiguousarray(b.T)).T if bt else dev(b)
    ta, tb = ta.to(dtype), tb.to(dtype)
    tc = dev(c0).to(dtype)
    lb.contract(ctx, alpha, (ta, "ik"), (tb, "kj"), beta, (tc, "ij"))
    got = to_np_f32(tc).astype(np.float64)
    an, bn, cn = to_np_f32(ta), to_np_f32(tb), to_np_f32(dev(c0).to(dtype))
    # exact (f64) product of the same rounded inputs, the accuracy reference
    exact = alpha * (an.astype(np.float64) @ bn.astype(np.float64))
    if beta != 0.0:
        exact = exact + beta * cn.astype(np.float64)
    if dtype == torch.bfloat16:
        exact = to_np_f32(torch.from_numpy(exact.astype(np.float32)).bfloat16()).astype(np.float64)
    denom = max(np.abs(exact).max(), 1e-30)
    rel = np.abs(got - exact).max() / denom
    # the CPU backend's sequential f32 product (crates/cpu/src/lib.rs:664-691) on the same inputs:
    # the GPU must sit within the tolerance plus the CPU's own rounding error of the exact value
    cpu = cn.copy()
    O.gemm3(O.DT_F32, O.DT_F32, O.DT_F32, an, bn, cpu, alpha, beta, threads=8)
    rel_cpu = np.abs(got - cpu).max() / denom
    cpu_err = np.abs(cpu - exact).max() / denom
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    assert rel_cpu <= tol + cpu_err, (rel_cpu, cpu_err)
    return rel, got, an, bn, cn


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (2, 2, 2), (5, 7, 11), (70, 50, 40), (33, 65, 1), (128, 256, 64),
                                   (129, 257, 100), (1024, 1024, 1024)])
def test_contract_f32_3xtf32(ctx, m, n, k):
    rel, got, a, b, c = run_gemm_case(ctx, m, n, k, seed=m + n + k)
    assert rel <= F32_TOL, rel
    # The reference's componentwise gate (K+2)u sum|a||b| assumes one f32 rounding per product;
    # 3xTF32 represents each operand to about 2^-22, so the gate applies from K = 16 on, where
    # the accumulation term dominates.
    if 16 <= k and m * n * k <= 1 << 22:
        assert gate_check(got, a, "ik", b, "kj", c, "ij", 1.0, 0.0) <= 1.0


def test_contract_f32_long_k_same_sign(ctx):
    """All-positive inputs make a truncating accumulation bias add up instead of cancelling:
    the chunked round-to-nearest accumulation must keep the f32 path within 1e-5 of exact."""
    for m, n, k in ((128, 128, 65536), (256, 256, 262144)):
        a = (data.uniform(41, (m, k)) + 1.0) * 0.5
        b = (data.uniform(42, (k, n)) + 1.0) * 0.5
        ta, tb = dev(a), dev(b)
        tc = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        lb.contract(ctx, 1.0, (ta, "ik"), (tb, "kj"), 0.0, (tc, "ij"))
        exact = (ta.double() @ tb.double()).cpu().numpy()
        rel = np.abs(tc.cpu().numpy() - exact).max() / np.abs(exact).max()
        assert rel <= F32_TOL, (m, n, k, rel)


@pytest.mark.parametrize("m,n,k", [(64, 64, 64), (200, 300, 1000), (1024, 1024, 1024), (64, 8192, 512)])
def test_contract_bf16(ctx, m, n, k):
    rel, *_ = run_gemm_case(ctx, m, n, k, dtype=torch.bfloat16, seed=7)
    assert rel <= BF16_TOL, rel


@pytest.mark.parametrize("m,n,k,bt,dtype", [(2304, 2304, 512, False, torch.bfloat16),
                                             (2400, 2560, 256, True, torch.bfloat16),
                                             (2560, 2304, 320, False, torch.float16)])
def test_contract_two_sm_tiles(ctx, m, n, k, bt, dtype):
    """Products with a 256 x 256 tile for every pair of SMs run on CTA pairs with cta_group::2
    MMAs (each CTA holds 128 rows of A and half of B^T): both B layouts, an M tail, f16.  f16
    products reach the tensor cores through the Backend slot's gemm (the op API rounds f16 once
    from a double-float dot instead)."""
    if dtype == torch.bfloat16:
        rel, *_ = run_gemm_case(ctx, m, n, k, dtype=dtype, bt=bt, seed=m + k)
        assert rel <= BF16_TOL, rel
    else:
        a = dev(data.uniform(m + k, (m, k))).half()
        b = dev(data.uniform(m + k + 1, (k, n))).half()
        c = torch.zeros(m, n, device="cuda", dtype=torch.float16)
        lb.backend_gemm(ctx, a, b, c, 1.0, 0.0)
        ctx.sync()
        exact = (a.double() @ b.double()).cpu().numpy()
        rel = np.abs(c.double().cpu().numpy() - exact).max() / np.abs(exact).max()
        assert rel <= BF16_TOL, rel
    assert "gemm_bf16_2sm_n256" in ctx.debug_launches()[-4:]


def test_contract_layouts_and_scalars(ctx):
    for at, bt in ((True, False), (False, True), (True, True)):
        rel, *_ = run_gemm_case(ctx, 96, 80, 72, at=at, bt=bt, seed=3)
        assert rel <= F32_TOL, (at, bt, rel)
    for beta in (0.0, 1.0, -0.5):
        for alpha in (1.0, -2.5):
            rel, *_ = run_gemm_case(ctx, 70, 50, 40, alpha=alpha, beta=beta, seed=11)
            assert rel <= F32_TOL, (alpha, beta, rel)
    # beta = 0 ignores NaN in C, alpha = 0 ignores NaN in A and B
    a = dev(np.array([[2.0, 3.0]], np.float32))
    b = dev(np.array([[4.0], [5.0]], np.float32))
    c = dev(np.array([[np.nan]], np.float32))
    lb.contract(ctx, 1.0, (a, "ik"), (b, "kj"), 0.0, (c, "ij"))
    assert c.item() == 23.0
    an = dev(np.full((1, 2), np.nan, np.float32))
    c2 = dev(np.array([[3.0, -4.0]], np.float32))
    lb.contract(ctx, 0.0, (an, "ik"), (dev(np.full((2, 2), np.nan, np.float32)), "kj"), 2.0, (c2, "ij"))
    assert c2.cpu().numpy().tolist() == [[6.0, -8.0]]


@pytest.mark.parametrize("m,n,k", [(1, 1, 1_000_003), (8, 8, 65_536), (3, 5, 200_001), (40, 24, 30_000),
                                   (1, 70, 9_973)])
def test_contract_split_k(ctx, m, n, k):
    rel, *_ = run_gemm_case(ctx, m, n, k, seed=1200 + m)
    assert rel <= F32_TOL, rel


def test_contract_batched_and_permuted(ctx):
    # batched long K (tests/contraction_test.rs:675-681 shape) with a transposed A
    a = data.uniform(1, (3, 50_000, 2))  # storage [b, k, m]; view bmk
    b = data.uniform(2, (3, 50_000, 4))
    c0 = data.uniform(3, (3, 2, 4))
    ta = dev(a).permute(0, 2, 1)
    tb, tc = dev(b), dev(c0)
    lb.contract(ctx, -1.0, (ta, "bmk"), (tb, "bkn"), 1.0, (tc, "bmn"))
    want = -np.einsum("bkm,bkn->bmn", a.astype(np.float64), b.astype(np.float64)) + c0
    rel = np.abs(tc.cpu().numpy() - want).max() / np.abs(want).max()
    assert rel <= F32_TOL
    # genuinely permuted contraction: A[32,8,16,24] over axes 1 and 3 (staged permute -> GEMM)
    a = data.uniform(4, (32, 8, 16, 24))
    b = data.uniform(5, (8, 24, 40))
    ta, tb = dev(a), dev(b)
    tc = torch.zeros((32, 16, 40), dtype=torch.float32, device="cuda")
    assert lb.plan_contract(ctx, 1.0, (ta, "abcd"), (tb, "bde"), 0.0, (tc, "ace"))["kind"] == "Staged"
    lb.contract(ctx, 1.0, (ta, "abcd"), (tb, "bde"), 0.0, (tc, "ace"))
    want = np.einsum("abcd,bde->ace", a.astype(np.float64), b.astype(np.float64))
    assert np.abs(tc.cpu().numpy() - want).max() / np.abs(want).max() <= F32_TOL


def test_contract_permuting_config_sampled(ctx):
    a = data.uniform(0, (32, 64, 128, 256))
    b = data.uniform(1, (128, 256, 512))
    ta, tb = dev(a), dev(b)
    tc = torch.zeros((32, 64, 512), dtype=torch.float32, device="cuda")
    lb.contract(ctx, 1.0, (ta, "abcd"), (tb, "cde"), 0.0, (tc, "abe"))
    got = tc.cpu().numpy().reshape(2048, 512)
    rng = np.random.default_rng(0)
    rows = rng.integers(0, 2048, 256)
    cols = rng.integers(0, 512, 256)
    cpu = O.gemm_entries(O.DT_F32, a.reshape(2048, 32768), b.reshape(32768, 512), 32768, rows, cols, n=512)
    rel = np.abs(got[rows, cols] - cpu).max() / np.abs(cpu).max()
    assert rel <= F32_TOL, rel


def test_contract_split_k_tall_bf16(ctx):
    K = 262144
    a = data.normal(0, (256, K), scale=K ** -0.5)
    b = data.normal(1, (K, 256), scale=K ** -0.5)
    ta, tb = dev(a).bfloat16(), dev(b).bfloat16()
    tc = torch.zeros((256, 256), dtype=torch.bfloat16, device="cuda")
    lb.contract(ctx, 1.0, (ta, "ik"), (tb, "kj"), 0.0, (tc, "ij"))
    ref = (ta.double() @ tb.double()).cpu().numpy()
    rel = np.abs(tc.float().cpu().numpy() - ref).max() / np.abs(ref).max()
    assert rel <= BF16_TOL, rel


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_contract_non_finite_inputs(ctx, dtype):
    """NaN and infinity reach exactly the outputs that depend on them, including through ragged
    boundary tiles and split-K (tests/contraction_test.rs:696-731): a NaN at A[m-1, k-1] and +inf
    at B[k/2, n-2].  The 3xTF32 path recomputes such units exactly; the other outputs keep the
    normwise tolerance against the f64 product of the finite inputs."""
    for seed, (m, n, k) in enumerate([(70, 45, 50), (3, 2, 40_000), (9, 11, 1), (300, 200, 4096)]):
        a = data.uniform(1400 + seed, (m, k))
        b = data.uniform(1450 + seed, (k, n))
        nan_row, inf_col = m - 1, n - 2
        a[nan_row, k - 1] = np.nan
        b[k // 2, inf_col] = np.inf
        ta, tb = dev(a).to(dtype), dev(b).to(dtype)
        c = torch.zeros((m, n), dtype=dtype, device="cuda")
        lb.contract(ctx, 1.0, (ta, "ik"), (tb, "kj"), 0.0, (c, "ij"))
        got = to_np_f32(c).astype(np.float64)
        an, bn = to_np_f32(ta).astype(np.float64), to_np_f32(tb).astype(np.float64)
        poisoned = np.zeros((m, n), bool)
        poisoned[nan_row, :] = True
        poisoned[:, inf_col] = True
        assert (np.isfinite(got) == ~poisoned).all(), np.argwhere(np.isfinite(got) == poisoned)[:5]
        assert np.isnan(got[nan_row, :]).all()
        rows = np.arange(m) != nan_row
        # an infinity times a nonzero finite a gives an infinity with a's sign (a is never 0 here)
        assert (got[rows, inf_col] == np.inf * np.sign(an[rows, k // 2])).all()
        af, bf = np.where(np.isfinite(an), an, 0.0), np.where(np.isfinite(bn), bn, 0.0)
        exact = af @ bf
        keep = ~poisoned
        denom = max(np.abs(exact[keep]).max(), 1e-30)
        rel = np.abs(got[keep] - exact[keep]).max() / denom
        assert rel <= (F32_TOL if dtype == torch.float32 else BF16_TOL), (m, n, k, rel)


def test_contract_determinism(ctx):
    a = dev(data.uniform(1300, (4, 300_000)))
    b = dev(data.uniform(1301, (300_000, 4)))
    outs = []
    for _ in range(3):
        c = torch.zeros((4, 4), dtype=torch.float32, device="cuda")
        lb.gemm(ctx, 1.0, a, b, 0.0, c)
        outs.append(bits(c))
    assert (outs[0] == outs[1]).all() and (outs[1] == outs[2]).all()


# ------------------------------------------------------------------------------------------------
# Backend training ops
# ------------------------------------------------------------------------------------------------

def test_bounded_wait_runs_out_and_context_recovers(gpu):
    """Failure detection without a GPU fault: a kernel waits, through the library's bounded wait,
    on a barrier nothing arrives on; after 50 ms it gives up and raises the device error word,
    lc_sync reports LC_ERR_DEVICE_TIMEOUT, and the same context then runs a product correctly."""
    c = lb.Context(0)
    c.debug_wait_probe(50_000)
    with pytest.raises(lb.DeviceTimeout):
        c.sync()
    c.sync()  # the error word was cleared
    a = torch.randn(256, 512, device="cuda")
    b = torch.randn(512, 128, device="cuda")
    out = torch.empty(256, 128, device="cuda")
    lb.contract(c, 1.0, (a, "ik"), (b, "kj"), 0.0, (out, "ij"))
    ref = a.double() @ b.double()
    assert ((out.double() - ref).abs().max() / ref.abs().max()).item() <= F32_TOL
    with pytest.raises(lb.InvalidArgument):
        c.debug_wait_probe(0)


def test_training_ops_match_oracle(ctx):
    x = data.normal(1, (37, 91))
    bvec = data.normal(2, (91,))
    tx, tb = dev(x), dev(bvec)
    ty = torch.empty_like(tx)
    lb.add_bias(ctx, tx, tb, ty)
    assert (bits(ty) == O.add_bias(x, bvec).view(np.uint32)).all()
    db = dev(data.normal(3, (91,)))
    db0 = db.cpu().numpy()
    lb.bias_grad(ctx, tx, db)
    assert (bits(db) == O.bias_grad(x, db0).view(np.uint32)).all()
    t = data.normal(4, (37, 91))
    tdy = torch.empty_like(tx)
    loss = lb.mse_grad(ctx, tx, dev(t), tdy)
    oloss, ody = O.mse_grad(x, t)
    assert (bits(tdy) == ody.view(np.uint32)).all()
    assert abs(loss - oloss) <= 1e-6 * abs(oloss)
    w = data.normal(5, (300,))
    g = data.normal(6, (300,))
    tw, tg = dev(w), dev(g)
    lb.sgd_step(ctx, tw, tg, 1e-3)
    ow, og = O.sgd_step(w, g, np.float32(1e-3))
    assert (bits(tw) == ow.view(np.uint32)).all() and (bits(tg) == 0).all()
    h = torch.empty(x.shape, dtype=torch.bfloat16, device="cuda")
    lb.convert(ctx, tx, h)
    assert (h.view(torch.int16).cpu().numpy().view(np.uint16) == O.f32_to_bf16(x)).all()
    back = torch.empty_like(tx)
    lb.convert(ctx, h, back)
    assert (bits(back) == O.bf16_to_f32(O.f32_to_bf16(x)).view(np.uint32)).all()
    lb.relu(ctx, tx, ty)
    assert (bits(ty) == O.relu(x).view(np.uint32)).all()
    lb.relu_backward(ctx, tx, dev(t), ty)
    assert (bits(ty) == O.relu_backward(x, t).view(np.uint32)).all()
    lb.gelu(ctx, tx, ty)
    assert np.abs(ty.cpu().numpy() - O.gelu(x)).max() <= 1e-6
    lb.gelu_backward(ctx, tx, dev(t), ty)
    assert np.abs(ty.cpu().numpy() - O.gelu_backward(x, t)).max() <= 1e-5


def test_backend_gemm_contract_rules(ctx):
    a = dev(data.uniform(1, (5, 7)))
    b = dev(data.uniform(2, (7, 3)))
    c = torch.zeros((5, 3), device="cuda")
    lb.backend_gemm(ctx, a, b, c, 1.0, 0.0)
    want = np.zeros((5, 3), np.float32)
    O.gemm(O.DT_F32, a.cpu().numpy(), b.cpu().numpy(), want, 1.0, 0.0)
    assert np.abs(c.cpu().numpy() - want).max() <= 1e-5 * np.abs(want).max()
    with pytest.raises(lb.ShapeError):
        lb.backend_gemm(ctx, a, a, c, 1.0, 0.0)
    with pytest.raises(lb.DtypeError):
        lb.backend_gemm(ctx, a, b.double(), c, 1.0, 0.0)
    with pytest.raises(lb.AliasError):
        lb.backend_gemm(ctx, a, b, lb.View.raw(a, 0, [5, 3], [3, 1]), 1.0, 0.0)
    with pytest.raises(lb.UnsupportedLayout):
        lb.backend_gemm(ctx, a, b, lb.View.raw(c, 1, [5, 3], [3, 1]), 1.0, 0.0)


# ------------------------------------------------------------------------------------------------
# f16: one rounding of a double-float dot (shaders/contraction.metal:445-755), bit-exact against
# the oracle's restatement
# ------------------------------------------------------------------------------------------------

def f16_bits(t) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("m,n,k,alpha,beta,at,bt", [(1, 1, 1, 1.0, 0.0, False, False), (37, 53, 300, 1.0, 0.0, False, False),
                                                    (64, 40, 1000, -0.75, 0.5, True, False),
                                                    (33, 17, 4097, 2.0, -1.0, False, True),
                                                    (300, 200, 64, 1.0, 1.0, True, True)])
def test_contract_f16_rounds_once_bit_exact(ctx, m, n, k, alpha, beta, at, bt):
    rng = np.random.default_rng(m * 7 + k)
    a = rng.standard_normal((k, m) if at else (m, k)).astype(np.float16)
    b = rng.standard_normal((n, k) if bt else (k, n)).astype(np.float16)
    c0 = rng.standard_normal((m, n)).astype(np.float16)
    ta = dev(a).t() if at else dev(a)
    tb = dev(b).t() if bt else dev(b)
    tc = dev(c0)
    assert lb.plan_contract(ctx, alpha, (ta, "ik"), (tb, "kj"), beta, (tc, "ij"))["kind"] == "General"
    lb.contract(ctx, alpha, (ta, "ik"), (tb, "kj"), beta, (tc, "ij"))
    want = c0.view(np.uint16).copy()
    O.contract_f16(a.view(np.uint16), b.view(np.uint16), want, alpha, beta,
                   a_strides=(1, m) if at else None, b_strides=(1, k) if bt else None, k=k)
    assert np.array_equal(f16_bits(tc), want)
    assert "contract_general_f16" in ctx.debug_launches()[-2:]


def test_contract_f16_multi_stride_in_place(ctx):
    """A permuted, batched f16 contraction (two strides per group) runs without staging copies
    and equals the oracle's per-batch products bit for bit."""
    rng = np.random.default_rng(9)
    a = rng.standard_normal((6, 8, 10, 12)).astype(np.float16)   # labels b m k1 k2 -> "bmcd"
    bm = rng.standard_normal((12, 6, 10, 7)).astype(np.float16)  # labels k2 b k1 n -> "dbce"
    ta, tb = dev(a), dev(bm)
    tc = torch.zeros((7, 6, 8), dtype=torch.float16, device="cuda")  # "ebm"
    plan = lb.plan_contract(ctx, 1.0, (ta, "bmcd"), (tb, "dbce"), 0.0, (tc, "ebm"))
    assert plan["kind"] == "General"
    lb.contract(ctx, 1.0, (ta, "bmcd"), (tb, "dbce"), 0.0, (tc, "ebm"))
    assert not any(n.startswith("strided_copy") or n.startswith("copy") for n in ctx.debug_launches()[-3:])
    got = f16_bits(tc)
    for bb in range(6):
        A = np.ascontiguousarray(a[bb].reshape(8, 120))                        # k = (c, d)
        B = np.ascontiguousarray(bm[:, bb].transpose(1, 0, 2).reshape(120, 7))  # k = (c, d)
        want = np.zeros((8, 7), np.uint16)
        O.contract_f16(A.view(np.uint16), B.view(np.uint16), want, 1.0, 0.0)
        assert np.array_equal(got[:, bb, :].T, want), bb


def test_contract_f16_scale_rounds_once(ctx):
    """tests/contraction_test.rs:445-470: K = 0 and beta = -0.999 take f16 0x0DDC to 0x8DDB."""
    a = torch.zeros((4, 0), dtype=torch.float16, device="cuda")
    b = torch.zeros((0, 3), dtype=torch.float16, device="cuda")
    c0 = np.random.default_rng(3).standard_normal((4, 3)).astype(np.float16)
    c0.view(np.uint16)[0, 0] = 0x0DDC
    c0[0, 1] = np.inf
    c0[0, 2] = np.nan
    tc = dev(c0)
    lb.contract(ctx, 1.0, (a, "ik"), (b, "kj"), -0.999, (tc, "ij"))
    got = f16_bits(tc)
    assert got[0, 0] == 0x8DDB and got[0, 1] == 0xFC00 and np.isnan(tc[0, 2].item())
    want = c0.view(np.uint16).copy()
    O.contract_f16(np.zeros((4, 0), np.uint16), np.zeros((0, 3), np.uint16), want, 1.0, -0.999, k=0)
    ok = (got == want) | (np.isnan(got.view(np.float16)) & np.isnan(want.view(np.float16)))
    assert ok.all()
