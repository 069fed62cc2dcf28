"""CPU-side checks of the C ABI: the library loads, exports every declared entry point, and its
host-only logic (schedule, placement, wire header, views, contraction planner) matches the
reference's rules and golden vectors.  No kernel is launched here."""
import json
import re
from pathlib import Path

import pytest

import linalg_b200 as lb
from oracle import oracle as O

ROOT = Path(__file__).resolve().parents[1]
G = json.loads((ROOT / "tests" / "golden" / "reference_goldens.json").read_text())


def declared_functions():
    names = []
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(lc_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    L = lb.load()
    names = declared_functions()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_local_order_matches_goldens_and_oracle():
    for c in G["local_order"]["cases"]:
        got = lb.local_order(c["stages"], c["rank"], c["m"])
        assert [f"{op}{m}" for op, m in got] == c["order"]
    for s, r, m in G["local_order"]["rejects"]:
        with pytest.raises(lb.ScheduleError):
            lb.local_order(s, r, m)
    for stages in range(1, 9):
        for rank in range(stages):
            for m in (1, 2, 5, 32):
                assert lb.local_order(stages, rank, m) == O.local_order(stages, rank, m)


def test_placement_matches_goldens():
    for layers, stages, owners in G["placement"]["cases"]:
        assert lb.contiguous_placement(layers, stages) == owners
    for layers, stages in G["placement"]["rejects"]:
        with pytest.raises(lb.ScheduleError):
            lb.contiguous_placement(layers, stages)
    assert lb.contiguous_placement(32, 8) == [r for r in range(8) for _ in range(4)]


def test_wire_header_matches_oracle_and_goldens():
    for c in G["wire"]["roundtrip"]:
        h = lb.wire_header(c["dtype"], c["shape"])
        assert h == O.wire_header(c["dtype"], c["shape"])
        payload = bytes.fromhex(c["payload"])
        assert lb.wire_parse(h + payload) == (c["dtype"], c["shape"], len(h))
    for c in G["wire"]["header_errors"]:
        exc = lb.ShapeError if c["error"] == "Shape" else lb.WireError
        with pytest.raises(exc):
            lb.wire_header(c["dtype"], c["shape"])
    good = lb.wire_header(1, [1]) + b"\x11\x22\x33\x44"
    for bad in (b"X" + good[1:], good[:16], good[:-1], good + b"\xff", b""):
        with pytest.raises(lb.WireError):
            lb.wire_parse(bad)


def _view(shape, strides=None, offset=0, dtype=lb.F32, nbytes=None, base=1 << 20):
    v = lb.lc_view()
    v.data = base
    v.offset = offset
    v.dtype = dtype
    v.rank = len(shape)
    if strides is None:
        strides, s = [], 1
        for n in reversed(shape):
            strides.insert(0, s)
            s *= n
    es = {lb.F32: 4, lb.BF16: 2, lb.F16: 2}[dtype]
    if nbytes is None:
        last = offset + sum((n - 1) * st for n, st in zip(shape, strides)) if all(shape) else offset
        nbytes = (last + 1) * es
    v.buffer_bytes = nbytes
    for i, (n, st) in enumerate(zip(shape, strides)):
        v.shape[i] = n
        v.strides[i] = st
    return lb.View(v, None)


def test_view_validate_and_slice_rules():
    L = lb.load()
    v = _view([64, 128, 128, 64])
    assert L.lc_view_validate(v.ref()) == 0
    s = lb.slice(v, [range(0, 64), range(32, 96), range(0, 128), range(16, 48)])
    assert s.offset == 32 * 8192 + 16 == 262160
    assert s.shape == [64, 64, 128, 32] and s.strides == [1048576, 8192, 64, 1]
    with pytest.raises(lb.InvalidArgument):
        lb.slice(v, [range(0, 65), range(0, 1), range(0, 1), range(0, 1)])
    with pytest.raises(lb.InvalidArgument):
        lb.slice(v, [range(0, 1)])
    short = _view([4], nbytes=12)
    assert L.lc_view_validate(short.ref()) == lb.ERR_INVALID_ARGUMENT
    p = lb.permute_view(v, [0, 3, 1, 2])
    assert p.shape == [64, 64, 128, 128] and p.strides == [1048576, 1, 8192, 64]
    with pytest.raises(lb.InvalidArgument):
        lb.permute_view(v, [0, 0, 1, 2])


def plan(a, al, b, bl, c, cl, alpha=1.0, beta=0.0):
    return lb.plan_contract(None, alpha, (a, al), (b, bl), beta, (c, cl))


def test_planner_baseline_configs():
    # 1024^3 f32: one tiled GEMM, no staging
    p = plan(_view([1024, 1024]), "ik", _view([1024, 1024], base=1 << 30), "kj", _view([1024, 1024], base=1 << 33), "ij")
    assert p["kind"] in ("Tiled", "Split") and (p["m"], p["n"], p["k"]) == (1024, 1024, 1024)
    assert p["a_major"] == "K" and p["b_major"] == "MN"
    # permuting config merges to M=2048, N=512, K=32768 with no staging
    a = _view([32, 64, 128, 256])
    b = _view([128, 256, 512], base=1 << 34)
    c = _view([32, 64, 512], base=1 << 36)
    p = plan(a, "abcd", b, "cde", c, "abe")
    assert (p["batch"], p["m"], p["n"], p["k"]) == (1, 2048, 512, 32768)
    assert p["kind"] in ("Tiled", "Split")
    # the genuinely permuted variant (A contracted over axes 1 and 3) stages A first
    b2 = _view([64, 256, 512], base=1 << 34)
    p = plan(a, "abcd", b2, "bde", _view([32, 128, 512], base=1 << 36), "ace")
    assert p["kind"] == "Staged" and (p["m"], p["n"], p["k"]) == (32 * 128, 512, 64 * 256)
    # split-K tall: 256 x 256 x 262144 splits
    p = plan(_view([256, 262144]), "ik", _view([262144, 256], base=1 << 34), "kj", _view([256, 256], base=1 << 36), "ij")
    assert p["kind"] == "Split" and p["splits"] > 1
    # skinny M swaps A and B
    p = plan(_view([64, 8192], dtype=lb.BF16), "ik", _view([8192, 8192], dtype=lb.BF16, base=1 << 34), "kj",
             _view([64, 8192], dtype=lb.BF16, base=1 << 36), "ij")
    assert p["swap_ab"]


def test_planner_scalar_rules_and_errors():
    a = _view([3, 4])
    b = _view([4, 5], base=1 << 30)
    c = _view([3, 5], base=1 << 31)
    assert plan(a, "ik", b, "kj", c, "ij", alpha=0.0)["kind"] == "Fill"
    assert plan(_view([3, 0]), "ik", _view([0, 5], base=1 << 30), "kj", c, "ij")["kind"] == "Fill"
    assert plan(_view([0, 4]), "ik", b, "kj", _view([0, 5], base=1 << 31), "ij")["kind"] == "Empty"
    with pytest.raises(lb.InvalidArgument):
        plan(a, "ik", b, "kj", c, "ix")  # label only in C
    with pytest.raises(lb.InvalidArgument):
        plan(a, "ii", b, "kj", c, "ij")  # repeated label
    with pytest.raises(lb.InvalidArgument):
        plan(a, "ik", _view([5, 5], base=1 << 30), "kj", c, "ij")  # extent mismatch
    with pytest.raises(lb.Overlap):
        plan(a, "ik", b, "kj", _view([3, 5], base=1 << 20), "ij")  # C overlaps A
    # C writing an element twice
    with pytest.raises(lb.Overlap):
        plan(a, "ik", b, "kj", _view([3, 5], strides=[0, 1], base=1 << 31), "ij")
