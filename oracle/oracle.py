"""ctypes front end of the CPU oracle (``liblinalg_oracle.so``).

TEST INFRASTRUCTURE ONLY: the checker for the GPU library and the timed CPU baseline.  The
product library never imports this module.  Each wrapper names the reference function it
restates; the C file cites the reference file:line for every algorithm.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liblinalg_oracle.so"

_u64 = C.c_uint64
_i64 = C.c_int64
_f32 = C.c_float
_f64 = C.c_double
_ptr = C.c_void_p

DT_F32, DT_F16, DT_BF16 = 1, 2, 3


def build() -> Path:
    """Compiles the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        sig = {
            "or_f32_to_bf16": (C.c_uint16, [_f32]),
            "or_bf16_to_f32": (_f32, [C.c_uint16]),
            "or_f32_to_f16": (C.c_uint16, [_f32]),
            "or_f16_to_f32": (_f32, [C.c_uint16]),
            "or_convert_f32_to_bf16": (None, [_ptr, _ptr, _u64]),
            "or_convert_bf16_to_f32": (None, [_ptr, _ptr, _u64]),
            "or_gemm": (C.c_int, [C.c_int, _u64, _u64, _u64, _f32, _f32, _ptr, _u64, _u64, _ptr, _u64, _u64,
                                  _ptr, _u64, _u64]),
            "or_gemm3": (C.c_int, [C.c_int, C.c_int, C.c_int, _u64, _u64, _u64, _f32, _f32, _ptr, _u64, _u64,
                                   _ptr, _u64, _u64, _ptr, _u64, _u64, C.c_int]),
            "or_gemm_entries": (None, [C.c_int, _u64, _f32, _ptr, _u64, _u64, _ptr, _u64, _u64, _ptr, _ptr,
                                       _u64, _ptr]),
            "or_contract_f64": (None, [_u64, _u64, _f64, _f64, _ptr, _u64, _ptr, _ptr, _ptr, _u64, _ptr, _ptr,
                                       _ptr, _ptr, _ptr, _ptr]),
            "or_gather": (None, [_ptr, _u64, _u64, C.c_int, _ptr, _ptr, _ptr]),
            "or_scatter": (None, [_ptr, _u64, _ptr, _u64, C.c_int, _ptr, _ptr]),
            "or_argmax": (_u64, [_ptr, _u64, _u64]),
            "or_argmax_rows": (None, [_ptr, _u64, _u64, _u64, _u64, _ptr]),
            "or_mag32": (_f32, [_f32, _f32, C.c_int]),
            "or_dd_to_f16": (C.c_uint16, [_f32, _f32]),
            "or_contract_f16": (None, [_u64, _u64, _u64, _f32, _f32, _ptr, _u64, _u64, _ptr, _u64, _u64, _ptr, _u64]),
            "or_argmax_complex": (_u64, [_ptr, _u64, _u64, C.c_int]),
            "or_sqrt": (None, [_ptr, _ptr, _u64]),
            "or_reciprocal": (None, [_ptr, _ptr, _u64]),
            "or_reciprocal_c32": (None, [_ptr, _ptr, _u64]),
            "or_add_bias": (None, [_ptr, _ptr, _ptr, _u64, _u64]),
            "or_bias_grad": (None, [_ptr, _ptr, _u64, _u64]),
            "or_mse_grad": (_f32, [_ptr, _ptr, _ptr, _u64]),
            "or_sgd_step": (None, [_ptr, _ptr, _u64, _f32]),
            "or_relu": (None, [_ptr, _ptr, _u64]),
            "or_relu_backward": (None, [_ptr, _ptr, _ptr, _u64]),
            "or_gelu": (None, [_ptr, _ptr, _u64]),
            "or_gelu_backward": (None, [_ptr, _ptr, _ptr, _u64]),
            "or_erf_constant_bits": (C.c_uint32, [C.c_int]),
            "or_local_order": (_i64, [_u64, _u64, _u64, _ptr]),
            "or_contiguous_placement": (C.c_int, [_u64, _u64, _ptr]),
            "or_wire_write_header": (_i64, [C.c_uint32, _ptr, C.c_uint32, _ptr, _ptr]),
            "or_wire_parse_header": (_i64, [_ptr, _u64, _ptr, _ptr, _ptr]),
            "or_train_reference": (C.c_int, [C.c_int, _u64, _ptr, _u64, _u64, _ptr, _ptr, _ptr, _ptr, _ptr]),
            "or_mlp_step": (_f32, [_u64, _u64, _u64, _u64, _f32, _ptr, _ptr, _ptr, C.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _u64arr(xs) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(list(xs), dtype=np.uint64))


# ---------------------------------------------------------------------------------------------
# conversions (crates/cpu/src/lib.rs:703-731)
# ---------------------------------------------------------------------------------------------

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    lib().or_convert_f32_to_bf16(_p(x), _p(y), x.size)
    return y


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    y = np.empty(h.shape, dtype=np.float32)
    lib().or_convert_bf16_to_f32(_p(h), _p(y), h.size)
    return y


def f32_to_f16_bits(v: float) -> int:
    return int(lib().or_f32_to_f16(float(np.float32(v))))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().or_f16_to_f32(h))


# ---------------------------------------------------------------------------------------------
# gemm (crates/cpu/src/lib.rs:203-295, :664-691)
# ---------------------------------------------------------------------------------------------

def gemm(dtype: int, a: np.ndarray, b: np.ndarray, c: np.ndarray, alpha: float, beta: float,
         a_strides=None, b_strides=None, threads: int = 1) -> np.ndarray:
    """``c = beta*c + alpha*a@b`` with the CPU backend's sequential k-order accumulate.

    a, b, c hold raw storage (float32 for f32, uint16 bits for f16/bf16).  ``a_strides`` /
    ``b_strides`` describe a transposed view (elements); default row-major.  c is updated
    in place and returned.
    """
    return gemm3(dtype, dtype, dtype, a, b, c, alpha, beta, a_strides, b_strides, threads)


def gemm3(adt: int, bdt: int, cdt: int, a, b, c, alpha, beta, a_strides=None, b_strides=None,
          threads: int = 1, shape=None):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert c.flags.c_contiguous
    m, n = c.shape
    if shape is not None:
        m, n, k = shape
    else:
        k = a.shape[1] if a_strides is None else a.shape[0]
    a_rs, a_cs = (k, 1) if a_strides is None else a_strides
    b_rs, b_cs = (n, 1) if b_strides is None else b_strides
    rc = lib().or_gemm3(adt, bdt, cdt, m, n, k, float(alpha), float(beta), _p(a), a_rs, a_cs, _p(b),
                        b_rs, b_cs, _p(c), n, 1, threads)
    if rc != 0:
        raise MemoryError("oracle gemm allocation failed")
    return c


def gemm_entries(dtype, a, b, k, rows, cols, alpha=1.0, a_strides=None, b_strides=None, n=None):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    rows = _u64arr(rows)
    cols = _u64arr(cols)
    out = np.empty(rows.size, dtype=np.float32)
    a_rs, a_cs = (k, 1) if a_strides is None else a_strides
    b_rs, b_cs = (n, 1) if b_strides is None else b_strides
    lib().or_gemm_entries(dtype, k, float(alpha), _p(a), a_rs, a_cs, _p(b), b_rs, b_cs, _p(rows), _p(cols),
                          rows.size, _p(out))
    return out


# ---------------------------------------------------------------------------------------------
# labelled contraction, f64 (tests/contraction_test.rs:202-262) and its accuracy gate (:283-313)
# ---------------------------------------------------------------------------------------------

def offset_table(labels: str, strides, over: str, extent: dict) -> np.ndarray:
    """tests/contraction_test.rs:202-222: element offsets of ``over`` labels in row-major order."""
    st = [strides[labels.index(l)] if l in labels else 0 for l in over]
    total = 1
    for l in over:
        total *= extent[l]
    if total == 0:
        return np.zeros(0, dtype=np.uint64)
    grids = np.indices([extent[l] for l in over], dtype=np.uint64).reshape(len(over), -1) if over else \
        np.zeros((0, 1), dtype=np.uint64)
    off = np.zeros(grids.shape[1], dtype=np.uint64)
    for d, s in enumerate(st):
        off += grids[d] * np.uint64(s)
    return np.ascontiguousarray(off)


def contract_reference(alpha, a_data, a_labels, a_off, a_shape, a_strides,
                       b_data, b_labels, b_off, b_shape, b_strides,
                       beta, c_data, c_labels, c_off, c_shape, c_strides):
    """Returns (exact f64 per output, magnitude per output, buffer index per output, K)."""
    extent = {}
    for labels, shape in ((a_labels, a_shape), (b_labels, b_shape), (c_labels, c_shape)):
        for l, n in zip(labels, shape):
            assert extent.setdefault(l, n) == n
    free = c_labels
    summed = "".join(l for l in a_labels if l in b_labels and l not in c_labels)
    a_free = offset_table(a_labels, a_strides, free, extent)
    a_sum = offset_table(a_labels, a_strides, summed, extent)
    b_free = offset_table(b_labels, b_strides, free, extent)
    b_sum = offset_table(b_labels, b_strides, summed, extent)
    idx = offset_table(c_labels, c_strides, free, extent) + np.uint64(c_off)
    a64 = np.ascontiguousarray(a_data, dtype=np.float64)
    b64 = np.ascontiguousarray(b_data, dtype=np.float64)
    c64 = np.ascontiguousarray(c_data, dtype=np.float64)
    n_out = idx.size
    exact = np.empty(n_out, dtype=np.float64)
    mag = np.empty(n_out, dtype=np.float64)
    n_sum = a_sum.size if summed else 1
    if not summed:
        a_sum = np.zeros(1, dtype=np.uint64)
        b_sum = np.zeros(1, dtype=np.uint64)
    lib().or_contract_f64(n_out, n_sum, float(alpha), float(beta), _p(a64), a_off, _p(a_free), _p(a_sum),
                          _p(b64), b_off, _p(b_free), _p(b_sum), _p(c64), _p(idx), _p(exact), _p(mag))
    return exact, mag, idx, int(np.prod([extent[l] for l in summed])) if summed else 1


U = 1.0 / 16777216.0


def contraction_gate(got: np.ndarray, exact: np.ndarray, magnitude: np.ndarray, k: int,
                     u_out: float = U, tiny: float = float(np.float32(1e-45))):
    """tests/contraction_test.rs:283-313: |C - C_ref| <= (K+2)u(|a||b|) + u_out|C_ref| + eta.

    Returns (worst err/tol, max err / (sqrt(K) u)).  ``got`` is float64 of the GPU output at
    the output indices; ``exact`` is rounded to the output type by the caller if desired."""
    rounded = exact.astype(np.float32).astype(np.float64) if u_out == U else exact
    err = np.abs(got - rounded)
    tol = (k + 2.0) * U * magnitude + u_out * np.abs(rounded) + tiny
    finite = np.isfinite(rounded)
    gate = float(np.max(err[finite] / tol[finite])) if finite.any() else 0.0
    norm = float(np.max(err[finite])) / (max(k, 1) ** 0.5 * U) if finite.any() else 0.0
    return gate, norm


# ---------------------------------------------------------------------------------------------
# permute / slice gathers (tests/permutation_test.rs:85-117, tests/slicing_test.rs:163-250)
# ---------------------------------------------------------------------------------------------

def gather(buf: np.ndarray, offset: int, shape, strides) -> np.ndarray:
    """Row-major copy of the strided view (raw element bits)."""
    buf = np.ascontiguousarray(buf)
    out = np.empty(tuple(shape), dtype=buf.dtype)
    rank = len(shape)
    lib().or_gather(_p(buf), buf.dtype.itemsize, offset, rank, _p(_u64arr(shape) if rank else _u64arr([1])),
                    _p(_u64arr(strides) if rank else _u64arr([0])), _p(out))
    return out


def scatter(src_logical: np.ndarray, dst_buf: np.ndarray, offset: int, shape, strides) -> np.ndarray:
    src = np.ascontiguousarray(src_logical)
    rank = len(shape)
    lib().or_scatter(_p(src), src.dtype.itemsize, _p(dst_buf), offset, rank,
                     _p(_u64arr(shape) if rank else _u64arr([1])), _p(_u64arr(strides) if rank else _u64arr([0])))
    return dst_buf


# ---------------------------------------------------------------------------------------------
# argmax / sqrt / reciprocal
# ---------------------------------------------------------------------------------------------

def argmax(x: np.ndarray, stride: int = 1, n: int | None = None) -> int:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size if n is None else n
    return int(lib().or_argmax(_p(x), n, stride))


def contract_f16(a_bits: np.ndarray, b_bits: np.ndarray, c_bits: np.ndarray, alpha: float, beta: float,
                 a_strides=None, b_strides=None, k: int | None = None) -> np.ndarray:
    """The op API's f16 product (shaders/contraction.metal:445-755): every output rounded once
    from a double-float dot.  Arrays hold f16 bits (uint16); c_bits [m, n] row-major is updated."""
    a = np.ascontiguousarray(a_bits, dtype=np.uint16)
    b = np.ascontiguousarray(b_bits, dtype=np.uint16)
    assert c_bits.dtype == np.uint16 and c_bits.flags.c_contiguous
    m, n = c_bits.shape
    if k is None:
        k = a.shape[1] if a_strides is None else a.shape[0]
    a_rs, a_cs = (k, 1) if a_strides is None else a_strides
    b_rs, b_cs = (n, 1) if b_strides is None else b_strides
    lib().or_contract_f16(m, n, k, float(np.float32(alpha)), float(np.float32(beta)), _p(a), a_rs, a_cs, _p(b), b_rs,
                          b_cs, _p(c_bits), n)
    return c_bits


MAG_L1, MAG_HYPOT = 0, 1


def mag32(re: float, im: float, kind: int) -> float:
    """tests/argmax_test.rs:51-72 `mag32`: the f32 complex magnitude the kernel ranks by."""
    return float(lib().or_mag32(float(np.float32(re)), float(np.float32(im)), kind))


def argmax_complex(z: np.ndarray, kind: int, stride: int = 1, n: int | None = None) -> int:
    """tests/argmax_test.rs:74-76 `ref_argmax_complex`; z is complex64 (or float32 pairs)."""
    z = np.ascontiguousarray(z)
    if z.dtype == np.complex64:
        z = z.view(np.float32)
    z = np.ascontiguousarray(z, dtype=np.float32).reshape(-1)
    n = z.size // 2 if n is None else n
    return int(lib().or_argmax_complex(_p(z), n, stride, kind))


def argmax_rows(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    cols = x.shape[-1]
    rows = x.size // cols
    out = np.empty(rows, dtype=np.uint32)
    lib().or_argmax_rows(_p(x), rows, cols, cols, 1, _p(out))
    return out.reshape(x.shape[:-1])


def sqrt(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().or_sqrt(_p(x), _p(y), x.size)
    return y


def reciprocal(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().or_reciprocal(_p(x), _p(y), x.size)
    return y


def reciprocal_c32(z: np.ndarray) -> np.ndarray:
    """1/z for complex f32 (re, im) pairs, bit for bit as shaders/reciprocal.metal:285-330."""
    z = np.ascontiguousarray(z, dtype=np.complex64)
    w = np.empty_like(z)
    lib().or_reciprocal_c32(_p(z), _p(w), z.size)
    return w


# ---------------------------------------------------------------------------------------------
# training ops (crates/cpu/src/lib.rs:372-533) and activations
# ---------------------------------------------------------------------------------------------

def add_bias(x, b):
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    y = np.empty_like(x)
    lib().or_add_bias(_p(x), _p(b), _p(y), x.shape[0], x.shape[1])
    return y


def bias_grad(dpre, db):
    dpre = np.ascontiguousarray(dpre, dtype=np.float32)
    db = np.ascontiguousarray(db, dtype=np.float32).copy()
    lib().or_bias_grad(_p(dpre), _p(db), dpre.shape[0], dpre.shape[1])
    return db


def mse_grad(y, t):
    y = np.ascontiguousarray(y, dtype=np.float32)
    t = np.ascontiguousarray(t, dtype=np.float32)
    dy = np.empty_like(y)
    loss = lib().or_mse_grad(_p(y), _p(t), _p(dy), y.size)
    return float(loss), dy


def sgd_step(w, dw, lr):
    w = np.ascontiguousarray(w, dtype=np.float32).copy()
    dw = np.ascontiguousarray(dw, dtype=np.float32).copy()
    lib().or_sgd_step(_p(w), _p(dw), w.size, float(lr))
    return w, dw


def relu(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().or_relu(_p(x), _p(y), x.size)
    return y


def relu_backward(pre, dy):
    pre = np.ascontiguousarray(pre, dtype=np.float32)
    dy = np.ascontiguousarray(dy, dtype=np.float32)
    dx = np.empty_like(pre)
    lib().or_relu_backward(_p(pre), _p(dy), _p(dx), pre.size)
    return dx


def gelu(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().or_gelu(_p(x), _p(y), x.size)
    return y


def gelu_backward(pre, dy):
    pre = np.ascontiguousarray(pre, dtype=np.float32)
    dy = np.ascontiguousarray(dy, dtype=np.float32)
    dx = np.empty_like(pre)
    lib().or_gelu_backward(_p(pre), _p(dy), _p(dx), pre.size)
    return dx


# ---------------------------------------------------------------------------------------------
# schedule / placement / wire (crates/schedule/src/lib.rs:15-35, crates/pipeline/src/lib.rs:29-40,
# crates/core/src/lib.rs:298-412)
# ---------------------------------------------------------------------------------------------

def local_order(stages: int, rank: int, microbatches: int):
    """Returns [("F", m) | ("B", m)] or None for Error::Schedule."""
    # microbatches > u32::MAX is rejected by the C side before it writes anything.
    cap = max(2 * microbatches, 1) if microbatches <= 0xFFFFFFFF else 1
    out = np.zeros(cap, dtype=np.int64)
    n = lib().or_local_order(stages, rank, microbatches, _p(out))
    if n < 0:
        return None
    return [("F", int(v) - 1) if v > 0 else ("B", int(-v) - 1) for v in out[:n]]


def contiguous_placement(layers: int, stages: int):
    out = np.zeros(max(layers, 1), dtype=np.uint64)
    if lib().or_contiguous_placement(layers, stages, _p(out)) != 0:
        return None
    return [int(v) for v in out[:layers]]


def wire_header(dtype_tag: int, shape) -> bytes:
    out = np.zeros(48, dtype=np.uint8)
    payload = np.zeros(1, dtype=np.uint64)
    sh = _u64arr(shape) if len(shape) else _u64arr([0])
    n = lib().or_wire_write_header(dtype_tag, _p(sh), len(shape), _p(out), _p(payload))
    if n < 0:
        raise ValueError({-1: "Wire", -2: "Shape"}[int(n)])
    return bytes(out[:n])


def wire_parse(msg: bytes):
    buf = np.frombuffer(msg, dtype=np.uint8).copy() if len(msg) else np.zeros(1, dtype=np.uint8)
    tag = np.zeros(1, dtype=np.uint32)
    shape = np.zeros(8, dtype=np.uint64)
    ndim = np.zeros(1, dtype=np.uint32)
    n = lib().or_wire_parse_header(_p(buf), len(msg), _p(tag), _p(shape), _p(ndim))
    if n < 0:
        raise ValueError({-1: "Wire", -2: "Shape"}[int(n)])
    return int(tag[0]), [int(v) for v in shape[: int(ndim[0])]], int(n)


# ---------------------------------------------------------------------------------------------
# pipeline references
# ---------------------------------------------------------------------------------------------

def train_reference(act: str, widths, batch: int, weights, xs, dys):
    """crates/pipeline/tests/pipeline.rs:396-480: sequential forward/backward, dW in microbatch
    order.  Returns (ys [mbs][batch][wL], dws list)."""
    layers = len(widths) - 1
    wcat = np.ascontiguousarray(np.concatenate([np.asarray(w, np.float32).ravel() for w in weights]))
    x = np.ascontiguousarray(np.stack([np.asarray(v, np.float32).reshape(batch, widths[0]) for v in xs]))
    dy = np.ascontiguousarray(np.stack([np.asarray(v, np.float32).reshape(batch, widths[-1]) for v in dys]))
    mbs = x.shape[0]
    y = np.zeros((mbs, batch, widths[-1]), dtype=np.float32)
    dw = np.zeros(wcat.size, dtype=np.float32)
    rc = lib().or_train_reference(0 if act == "gelu" else 1, layers, _p(_u64arr(widths)), batch, mbs, _p(wcat),
                                  _p(x), _p(dy), _p(y), _p(dw))
    assert rc == 0
    out, o = [], 0
    for l in range(layers):
        n = widths[l] * widths[l + 1]
        out.append(dw[o:o + n].reshape(widths[l], widths[l + 1]))
        o += n
    return y, out


def mlp_step(master: np.ndarray, x: np.ndarray, t: np.ndarray, microbatch: int, lr: float,
             threads: int = 1) -> float:
    """One benchmark training step (see or_mlp_step); ``master`` [L, d, d] is updated in place."""
    assert master.dtype == np.float32 and master.flags.c_contiguous
    layers, d, _ = master.shape
    x = np.ascontiguousarray(x, dtype=np.float32)
    t = np.ascontiguousarray(t, dtype=np.float32)
    return float(lib().or_mlp_step(layers, d, x.shape[0], microbatch, float(lr), _p(master), _p(x), _p(t),
                                   threads))
