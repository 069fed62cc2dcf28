"""Pins the CPU oracle to the reference's own known-answer tests (tests/golden).

The reference (Rust + Metal) cannot be built in this container, so these vectors, read out of
its test sources, are what ties the oracle restatement to the reference's behaviour.
"""
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

G = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())


def f32(bits: str) -> np.float32:
    return np.frombuffer(struct.pack("<I", int(bits, 16)), dtype=np.float32)[0]


def bits_of(x) -> int:
    return int(np.asarray(x, dtype=np.float32).view(np.uint32))


def arr(case, key):
    if key + "_bits" in case:
        return np.array([f32(b) for b in case[key + "_bits"]], dtype=np.float32)
    return np.array(case.get(key, []), dtype=np.float32)


@pytest.mark.parametrize("case", G["gemm_f32"], ids=lambda c: c["cite"].split(" ")[0])
def test_gemm_f32_goldens(case):
    m, n, k = case["m"], case["n"], case["k"]
    a = arr(case, "a").reshape(m, k)
    b = arr(case, "b").reshape(k, n)
    c = arr(case, "c0").reshape(m, n).copy()
    c0 = c.copy()
    alpha, beta = np.float32(case["alpha"]), np.float32(case["beta"])
    O.gemm(O.DT_F32, a, b, c, alpha, beta)
    if "expected" in case:
        assert [bits_of(v) for v in c.ravel()] == [bits_of(v) for v in np.float32(case["expected"])]
    if "expected_bits" in case:
        assert [bits_of(v) for v in c.ravel()] == [int(x, 16) for x in case["expected_bits"]]
    if case.get("expected_c00_formula"):
        acc = np.float32(beta * c0[0, 0])
        acc = np.float32(acc + np.float32(np.float32(alpha * a[0, 0]) * b[0, 0]))
        acc = np.float32(acc + np.float32(np.float32(alpha * a[0, 1]) * b[1, 0]))
        assert bits_of(c[0, 0]) == bits_of(acc)
    if case.get("expected_left_assoc"):
        left = np.float32(np.float32(alpha * a[0, 0]) * b[0, 0])
        right = np.float32(alpha * np.float32(a[0, 0] * b[0, 0]))
        assert bits_of(left) != bits_of(right)
        assert bits_of(c[0, 0]) == bits_of(left)


def test_gemm_transposed_layouts_match_row_major():
    # crates/cpu/src/invariants.rs:100-134: the three layouts give the same bits.
    rng = np.random.default_rng(3)
    m, n, k = 5, 7, 11
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    ref = np.zeros((m, n), np.float32)
    O.gemm(O.DT_F32, a, b, ref, 1.0, 0.0)
    at = np.ascontiguousarray(a.T)  # storage [k, m]; the view has strides [1, m]
    c1 = np.zeros((m, n), np.float32)
    O.gemm(O.DT_F32, at, b, c1, 1.0, 0.0, a_strides=(1, m))
    bt = np.ascontiguousarray(b.T)
    c2 = np.zeros((m, n), np.float32)
    O.gemm(O.DT_F32, a, bt, c2, 1.0, 0.0, b_strides=(1, k))
    assert (ref.view(np.uint32) == c1.view(np.uint32)).all()
    assert (ref.view(np.uint32) == c2.view(np.uint32)).all()


def test_half_conversions():
    h = G["half_conversions"]
    for v, bits in h["f16"]:
        assert O.f32_to_f16_bits(v) == int(bits, 16)
    for v, bits in h["bf16"]:
        assert int(O.f32_to_bf16(np.float32([v]))[0]) == int(bits, 16)


@pytest.mark.parametrize("case", G["gemm_half"]["cases"])
def test_gemm_half_goldens(case):
    dt = O.DT_F16 if case["dtype"] == "f16" else O.DT_BF16

    def enc(vals):
        if dt == O.DT_F16:
            return np.array([O.f32_to_f16_bits(v) for v in vals], dtype=np.uint16)
        return O.f32_to_bf16(np.float32(vals))

    k = len(case["a"])
    a = enc(case["a"]).reshape(1, k)
    b = enc(case["b"]).reshape(k, 1)
    c = enc(case["c"]).reshape(1, 1).copy()
    O.gemm(dt, a, b, c, case["alpha"], case["beta"])
    assert int(c[0, 0]) == int(case["expected"], 16)


def test_convert_f32_to_bf16_goldens():
    cv = G["convert_f32_to_bf16"]
    xs = np.array([f32(a) for a, _ in cv["cases"]], dtype=np.float32)
    got = O.f32_to_bf16(xs)
    assert [int(v) for v in got] == [int(b, 16) for _, b in cv["cases"]]
    nans = np.array([f32(b) for b in cv["nan_inputs"]], dtype=np.float32)
    for bits, g in zip(cv["nan_inputs"], O.f32_to_bf16(nans)):
        g = int(g)
        assert g & 0x7F80 == 0x7F80 and g & 0x007F != 0
        assert g & 0x0040
        assert g & 0x8000 == (int(bits, 16) >> 16) & 0x8000
    allh = np.arange(65536, dtype=np.uint16)
    back = O.bf16_to_f32(allh)
    assert (back.view(np.uint32) == (allh.astype(np.uint32) << 16)).all()


def test_sgd_step_bits():
    # crates/cpu/src/training.rs:203-218
    rng = np.random.default_rng(7)
    w = rng.standard_normal(300).astype(np.float32)
    g = rng.standard_normal(300).astype(np.float32)
    lr = np.float32(1e-3)
    w2, g2 = O.sgd_step(w, g, lr)
    want = (w - (lr * g).astype(np.float32)).astype(np.float32)
    assert (w2.view(np.uint32) == want.view(np.uint32)).all()
    assert (g2.view(np.uint32) == 0).all()


def test_mse_grad_matches_sequential_definition():
    rng = np.random.default_rng(8)
    y = rng.standard_normal(97).astype(np.float32)
    t = rng.standard_normal(97).astype(np.float32)
    loss, dy = O.mse_grad(y, t)
    s = np.float32(0)
    n = np.float32(97)
    for i in range(97):
        d = np.float32(y[i] - t[i])
        s = np.float32(s + np.float32(d * d))
        assert bits_of(dy[i]) == bits_of(np.float32(np.float32(2 * d) / n))
    assert bits_of(np.float32(loss)) == bits_of(np.float32(s / n))


def test_erf_constants():
    assert [O.lib().or_erf_constant_bits(i) for i in range(6)] == [int(b, 16) for b in G["erf_constants"]["bits"]]


def test_local_order_goldens():
    lo = G["local_order"]
    for c in lo["cases"]:
        got = O.local_order(c["stages"], c["rank"], c["m"])
        assert [f"{op}{m}" for op, m in got] == c["order"]
    for s, r, m in lo["rejects"]:
        assert O.local_order(s, r, m) is None


def test_local_order_properties():
    # crates/schedule/src/lib.rs:113-180
    for stages in range(1, 6):
        for rank in range(stages):
            for m in range(1, 9):
                order = O.local_order(stages, rank, m)
                fs = [i for op, i in order if op == "F"]
                bs = [i for op, i in order if op == "B"]
                assert fs == list(range(m)) and bs == list(range(m))
                for mb in range(m):
                    assert order.index(("F", mb)) < order.index(("B", mb))


def test_placement_goldens():
    p = G["placement"]
    for layers, stages, owners in p["cases"]:
        assert O.contiguous_placement(layers, stages) == owners
    for layers, stages in p["rejects"]:
        assert O.contiguous_placement(layers, stages) is None


@pytest.mark.parametrize("case", G["argmax"]["cases"])
def test_argmax_goldens(case):
    x = arr(case, "x")
    assert O.argmax(x) == case["expected"]


def complex_case(case) -> np.ndarray:
    """The n complex values of a transcribed argmax_complex case (interleaved f32 pairs)."""
    z = np.empty((case["n"], 2), np.float32)
    z[:, 0] = f32(case["fill"][0])
    z[:, 1] = f32(case["fill"][1])
    for i, re, im in case["set"]:
        z[i] = (f32(re), f32(im))
    return z


@pytest.mark.parametrize("case", G["argmax_complex"]["cases"])
def test_argmax_complex_goldens(case):
    z = complex_case(case)
    for kind, want in case["expected"].items():
        assert O.argmax_complex(z, O.MAG_L1 if kind == "l1" else O.MAG_HYPOT) == want, (case["cite"], kind)


def test_mag32_formulas():
    # tests/argmax_test.rs:51-72: NaN parts give NaN, hi == 0 gives 0, an infinite part gives inf,
    # and the scaled hypot stays finite where re^2 + im^2 would overflow
    assert np.isnan(O.mag32(np.nan, 1.0, O.MAG_HYPOT)) and np.isnan(O.mag32(1.0, np.nan, O.MAG_L1))
    assert O.mag32(-0.0, 0.0, O.MAG_HYPOT) == 0.0
    assert O.mag32(np.inf, np.nan, O.MAG_L1) != O.mag32(np.inf, np.nan, O.MAG_L1)
    assert O.mag32(np.inf, 3.0, O.MAG_HYPOT) == np.inf
    assert O.mag32(3.0, -4.0, O.MAG_HYPOT) == 5.0 and O.mag32(3.0, -4.0, O.MAG_L1) == 7.0
    big = float(np.float32(2e38))  # hypot 2.83e38: finite, while big * big overflows
    assert np.isfinite(O.mag32(big, big, O.MAG_HYPOT))


def test_argmax_nan_and_ties():
    # tests/argmax_test.rs:316-362 style cases
    x = np.ones(10, np.float32)
    x[3] = np.inf
    x[7] = np.nan
    assert O.argmax(x) == 7
    x[1] = -np.nan
    assert O.argmax(x) == 1
    y = np.full(9, 7.0, np.float32)
    y[::2] = -7.0
    assert O.argmax(y) == 0


def test_sqrt_and_reciprocal_goldens():
    for xb, yb in G["sqrt"]["cases"]:
        assert bits_of(O.sqrt(np.array([f32(xb)]))[0]) == int(yb, 16)
    s = G["reciprocal"]["simple"]
    assert list(O.reciprocal(np.float32(s["x"]))) == s["y"]
    xs = np.array([f32(a) for a, _ in G["reciprocal"]["cases"]], np.float32)
    assert [bits_of(v) for v in O.reciprocal(xs)] == [int(b, 16) for _, b in G["reciprocal"]["cases"]]


def c32_of(pair) -> np.complex64:
    return np.array([int(pair[0], 16), int(pair[1], 16)], np.uint32).view(np.complex64)[0]


def test_complex_reciprocal_goldens():
    """Every exact complex result the reference's reciprocal tests assert, and the NaN rule."""
    g = G["reciprocal_c32"]
    zs = np.array([c32_of(e["z"]) for e in g["exact"]], np.complex64)
    ws = O.reciprocal_c32(zs).view(np.uint32).reshape(-1, 2)
    for e, w in zip(g["exact"], ws):
        assert [int(w[0]), int(w[1])] == [int(e["w"][0], 16), int(e["w"][1], 16)], e
    nz = np.array([c32_of(p) for p in g["nan_inputs"]], np.complex64)
    assert (O.reciprocal_c32(nz).view(np.uint32) == 0x7FC00000).all()


def fields_to_f32(rng, fields):
    """Random-signed floats whose magnitudes lie in [2^(f-127), 2^(f-126)) for biased exponent
    field f, extended below 1 to subnormals (tests/reciprocal_test.rs:264-278, own generator)."""
    fields = np.asarray(fields, np.int64)
    frac = rng.integers(0, 1 << 23, size=fields.shape, dtype=np.int64)
    top = np.left_shift(1, np.clip(22 + fields, 0, 22))
    mag = np.where(fields >= 1, (np.clip(fields, 1, 254) << 23) | frac, top | (frac & (top - 1)))
    sign = rng.integers(0, 2, size=fields.shape, dtype=np.int64) << 31
    return (mag | sign).astype(np.uint32).view(np.float32)


def complex_inputs(seed, count, lo, hi, spread):
    rng = np.random.default_rng(seed)
    re = rng.integers(lo, hi + 1, size=count)
    im = rng.integers(np.maximum(lo, re - spread), np.minimum(hi, re + spread) + 1)
    z = np.empty(count, np.complex64)
    z.real, z.imag = fields_to_f32(rng, re), fields_to_f32(rng, im)
    return z


def ulp_distance(got: np.ndarray, want: np.ndarray) -> np.ndarray:
    """f32 distance with infinity next to the largest finite value; NaN matches only NaN and
    the signs (zero's too) must agree, else a huge distance (tests/reciprocal_test.rs:148-158)."""
    gb, wb = got.view(np.uint32).astype(np.int64), want.view(np.uint32).astype(np.int64)
    d = np.abs((gb & 0x7FFFFFFF) - (wb & 0x7FFFFFFF))
    both_nan = np.isnan(got) & np.isnan(want)
    bad = (np.isnan(got) != np.isnan(want)) | ((gb >> 31) != (wb >> 31))
    return np.where((gb == wb) | both_nan, 0, np.where(bad, 1 << 40, d))


def assert_complex_gate(z: np.ndarray, w: np.ndarray):
    """The reference's accuracy gate for finite nonzero z (tests/reciprocal_test.rs:187-229):
    normwise error <= 4u |1/z| + 2^-149 against the f64 value, each part within 4 ulps of it."""
    a, b = z.real.astype(np.float64), z.imag.astype(np.float64)
    n2 = a * a + b * b
    want = [a / n2, -b / n2]
    got = [w.real, w.imag]
    delta, ulps = [], np.zeros(len(z), np.int64)
    for c in range(2):
        with np.errstate(over="ignore"):  # results past the f32 range round to infinity
            rounded = want[c].astype(np.float32)
        ulps = np.maximum(ulps, ulp_distance(got[c], rounded))
        g = got[c].astype(np.float64)
        delta.append(np.where(~np.isinf(g), g - want[c],
                              np.where(np.isinf(rounded), 0.0, np.copysign(2.0 ** 128, g) - want[c])))
    absolute = np.hypot(delta[0], delta[1])
    modulus = np.hypot(want[0], want[1])
    ok = (ulps <= 4) & (absolute <= 4.0 * 2.0 ** -24 * modulus + 2.0 ** -149)
    assert ok.all(), (z[~ok][:4], w[~ok][:4])


@pytest.mark.parametrize("seed,lo,hi,spread", [(10, 87, 167, 80), (11, 87, 167, 2), (12, -22, 254, 276),
                                               (20, 245, 254, 9), (30, -22, 3, 25), (31, -22, 60, 82)])
def test_complex_reciprocal_oracle_meets_gate(seed, lo, hi, spread):
    """The restatement meets the reference's accuracy gate on the input families of its tests
    (moderate, comparable parts, full range, near overflow, near underflow)."""
    z = complex_inputs(seed, 20_000, lo, hi, spread)
    assert_complex_gate(z, O.reciprocal_c32(z))


def test_wire_goldens():
    w = G["wire"]
    for c in w["roundtrip"]:
        payload = bytes.fromhex(c["payload"])
        msg = O.wire_header(c["dtype"], c["shape"]) + payload
        assert msg[:4] == b"LNGL"
        tag, shape, off = O.wire_parse(msg)
        assert (tag, shape, msg[off:]) == (c["dtype"], c["shape"], payload)
    for c in w["lengths"]:
        nbytes = 4 if c["dtype"] == 1 else 2
        for s in c["shape"]:
            nbytes *= s
        assert len(O.wire_header(c["dtype"], c["shape"])) + nbytes == c["len"]
    for c in w["header_errors"]:
        with pytest.raises(ValueError, match=c["error"]):
            O.wire_header(c["dtype"], c["shape"])
    good = O.wire_header(1, [1]) + b"\x11\x22\x33\x44"
    for bad in (b"X" + good[1:], good[:4] + struct.pack("<I", 2) + good[8:], b"", b"\0" * 15, good[:16],
                good[:-1], good + b"\xff"):
        with pytest.raises(ValueError, match="Wire"):
            O.wire_parse(bad)


def _fixture_weights():
    fx = G["pipeline_fixture"]
    widths = fx["widths"]
    ws = []
    for l in range(len(widths) - 1):
        w = np.zeros((widths[l], widths[l + 1]), np.float32)
        for r in range(widths[l]):
            for c in range(widths[l + 1]):
                v = np.float32(np.float32(0.1) * np.float32(r + 1)) - np.float32(np.float32(0.05) * np.float32(c + 1))
                w[r, c] = np.float32(np.float32(v) + np.float32(np.float32(0.02) * np.float32(l)))
        ws.append(w)
    return fx, widths, ws


def test_train_reference_matches_hand_sequential():
    """crates/pipeline/tests/pipeline.rs:396-480: the sequential reference over the tiny fixture,
    restated with numpy f32 ops in the same order, equals the C restatement bit for bit."""
    fx, widths, ws = _fixture_weights()
    b = fx["batch"]
    xs = [fx["x0"], fx["x1"]]
    dys = [fx["dy0"], fx["dy1"]]
    y, dw = O.train_reference("gelu", widths, b, ws, xs, dys)
    # independent restatement with the oracle's gemm and gelu pieces, microbatch by microbatch
    dws = [np.zeros_like(w) for w in ws]
    for mb in range(2):
        acts = [np.float32(xs[mb]).reshape(b, widths[0])]
        pres = []
        for l, w in enumerate(ws):
            pre = np.zeros((b, widths[l + 1]), np.float32)
            O.gemm(O.DT_F32, acts[-1], w, pre, 1.0, 0.0)
            pres.append(pre)
            acts.append(O.gelu(pre))
        assert (acts[-1].view(np.uint32) == y[mb].view(np.uint32)).all()
        g = np.float32(dys[mb]).reshape(b, widths[-1])
        for l in reversed(range(len(ws))):
            dpre = O.gelu_backward(pres[l], g)
            O.gemm(O.DT_F32, np.ascontiguousarray(acts[l].T), dpre, dws[l], 1.0, 1.0)
            dx = np.zeros((b, widths[l]), np.float32)
            O.gemm(O.DT_F32, dpre, np.ascontiguousarray(ws[l].T), dx, 1.0, 0.0)
            g = dx
    for got, want in zip(dw, dws):
        assert (got.view(np.uint32) == want.view(np.uint32)).all()


def test_mlp_step_decreases_loss_and_is_thread_invariant():
    rng = np.random.default_rng(11)
    L, d, B, mb = 2, 32, 16, 4
    master = (rng.standard_normal((L, d, d)) / np.sqrt(d)).astype(np.float32)
    x = rng.standard_normal((B, d)).astype(np.float32)
    t = rng.standard_normal((B, d)).astype(np.float32)
    m1 = master.copy()
    m2 = master.copy()
    l1 = O.mlp_step(m1, x, t, mb, 0.5, threads=1)
    l2 = O.mlp_step(m2, x, t, mb, 0.5, threads=3)
    assert l1 == l2 and (m1.view(np.uint32) == m2.view(np.uint32)).all()
    l3 = O.mlp_step(m1, x, t, mb, 0.5, threads=1)
    assert l3 < l1


def test_f16_scale_rounds_once_golden():
    g = G["contract_f16_scale"]
    for cin, cout in g["cases"]:
        c = np.array([[int(cin, 16)]], np.uint16)
        O.contract_f16(np.zeros((1, 0), np.uint16), np.zeros((0, 1), np.uint16), c, 1.0, g["beta"], k=0)
        assert int(c[0, 0]) == int(cout, 16), (cin, hex(int(c[0, 0])))


def test_f16_contraction_is_the_correctly_rounded_dot():
    """A double-float dot of exact f16 products, rounded once, is the correctly rounded f16 of
    the exact sum (the f64 sum of these products is exact to far below an f16 half-ulp), which is
    what the reference's gate expects of f16 outputs (tests/contraction_test.rs:1-13)."""
    rng = np.random.default_rng(16)
    for m, n, k, alpha, beta in ((7, 9, 33, 1.0, 0.0), (16, 5, 1000, -0.5, 0.0), (4, 4, 257, 2.0, 1.0)):
        a = rng.standard_normal((m, k)).astype(np.float16)
        b = rng.standard_normal((k, n)).astype(np.float16)
        c0 = rng.standard_normal((m, n)).astype(np.float16)
        c = c0.view(np.uint16).copy()
        O.contract_f16(a.view(np.uint16), b.view(np.uint16), c, alpha, beta)
        exact = alpha * (a.astype(np.float64) @ b.astype(np.float64)) + beta * c0.astype(np.float64)
        assert np.array_equal(c, exact.astype(np.float16).view(np.uint16)), (m, n, k)
