"""Python front end of ``liblinalg_b200.so`` (the C ABI in include/linalg_b200.h).

The functions mirror the reference's Rust op API (src/ops/*.rs) by name, argument meaning
and error behaviour: ``contract`` / ``encode_contract``, ``gemm`` / ``encode_gemm``,
``permute_view``, ``materialize``, ``conjugate``, ``adjoint``, ``slice``, ``pack``,
``concat``, ``argmax``, ``argmax_complex``, ``sqrt``, ``reciprocal``; plus the ``Backend``
training ops and the 1F1B pipeline.  Device memory comes from torch tensors (torch is only
the allocator and stream source here); every computation runs in the CUDA library, and
importing this module on a machine without the built library or without a B200 raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liblinalg_b200.so"
MAX_RANK = 8

# status codes (include/linalg_b200.h)
OK = 0
ERR_NO_DEVICE, ERR_INVALID_ARGUMENT, ERR_OVERLAP, ERR_LAUNCH = 1, 2, 3, 4
ERR_SHAPE, ERR_DTYPE, ERR_UNSUPPORTED_LAYOUT, ERR_UNSUPPORTED_DEVICE = 10, 11, 12, 13
ERR_ALIAS, ERR_TRANSPORT, ERR_WIRE, ERR_SCHEDULE = 14, 15, 16, 17
ERR_CUDA, ERR_DEVICE_TIMEOUT = 20, 21

F32, F16, BF16, U32, I32, C32, F64, C64, U16 = 1, 2, 3, 4, 5, 6, 7, 8, 9


class LinalgError(RuntimeError):
    """Base of every error the library reports; ``code`` is the lc_status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class NoDevice(LinalgError): pass
class InvalidArgument(LinalgError): pass
class Overlap(LinalgError): pass
class LaunchError(LinalgError): pass
class ShapeError(LinalgError): pass
class DtypeError(LinalgError): pass
class UnsupportedLayout(LinalgError): pass
class AliasError(LinalgError): pass
class TransportError(LinalgError): pass
class WireError(LinalgError): pass
class ScheduleError(LinalgError): pass
class CudaError(LinalgError): pass
class DeviceTimeout(LinalgError): pass


_ERRORS = {ERR_NO_DEVICE: NoDevice, ERR_INVALID_ARGUMENT: InvalidArgument, ERR_OVERLAP: Overlap,
           ERR_LAUNCH: LaunchError, ERR_SHAPE: ShapeError, ERR_DTYPE: DtypeError,
           ERR_UNSUPPORTED_LAYOUT: UnsupportedLayout, ERR_ALIAS: AliasError, ERR_TRANSPORT: TransportError,
           ERR_WIRE: WireError, ERR_SCHEDULE: ScheduleError, ERR_CUDA: CudaError,
           ERR_DEVICE_TIMEOUT: DeviceTimeout}


class lc_view(C.Structure):
    _fields_ = [("data", C.c_void_p), ("buffer_bytes", C.c_uint64), ("offset", C.c_uint64),
                ("dtype", C.c_int32), ("rank", C.c_int32), ("shape", C.c_uint64 * MAX_RANK),
                ("strides", C.c_uint64 * MAX_RANK)]


class lc_contract_plan(C.Structure):
    _fields_ = [("kind", C.c_int32), ("splits", C.c_int32), ("batch", C.c_uint64), ("m", C.c_uint64),
                ("n", C.c_uint64), ("k", C.c_uint64), ("swap_ab", C.c_int32), ("a_major", C.c_int32),
                ("b_major", C.c_int32)]


class lc_epilogue(C.Structure):
    _fields_ = [("kind", C.c_int32), ("aux", C.c_void_p), ("aux2", C.c_void_p), ("lr", C.c_float),
                ("tile_n", C.c_int32), ("splits", C.c_int32), ("swap", C.c_int32)]


EPI_NONE, EPI_RELU, EPI_RELU_MASK, EPI_SGD, EPI_GELU, EPI_GELU_BACKWARD = 0, 1, 2, 3, 4, 5


class lc_pipeline_config(C.Structure):
    _fields_ = [("layers", C.c_uint64), ("width", C.c_uint64), ("widths", C.POINTER(C.c_uint64)),
                ("microbatch", C.c_uint64),
                ("microbatches", C.c_uint64), ("activation", C.c_int32), ("compute_dtype", C.c_int32),
                ("lr", C.c_float), ("loss", C.c_int32), ("timeout_ms", C.c_int32)]


_lib = None
_V = C.POINTER(lc_view)
_vp = C.c_void_p


def _sig(L):
    s = C.c_int32
    f = C.c_float
    table = {
        "lc_context_create": (s, [C.c_int, C.POINTER(_vp)]),
        "lc_context_destroy": (s, [_vp]),
        "lc_context_stream": (_vp, [_vp]),
        "lc_sync": (s, [_vp, _vp]),
        "lc_last_error": (C.c_char_p, []),
        "lc_debug_launches": (C.c_uint64, [_vp]),
        "lc_debug_launch_name": (C.c_char_p, [_vp, C.c_uint64]),
        "lc_debug_wait_probe": (C.c_int, [_vp, _vp, C.c_uint32]),
        "lc_view_validate": (s, [_V]),
        "lc_permute_view": (s, [_V, C.POINTER(C.c_int32), C.c_int32, _V]),
        "lc_slice": (s, [_V, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.c_int32, _V]),
        "lc_encode_contract": (s, [_vp, _vp, f, _V, C.c_char_p, _V, C.c_char_p, f, _V, C.c_char_p]),
        "lc_contract": (s, [_vp, f, _V, C.c_char_p, _V, C.c_char_p, f, _V, C.c_char_p]),
        "lc_plan_contract": (s, [_vp, f, _V, C.c_char_p, _V, C.c_char_p, f, _V, C.c_char_p,
                                 C.POINTER(lc_contract_plan)]),
        "lc_encode_gemm": (s, [_vp, _vp, f, _V, _V, f, _V]),
        "lc_gemm": (s, [_vp, f, _V, _V, f, _V]),
        "lc_encode_gemm_noalloc": (s, [_vp, _vp, f, _V, _V, f, _V]),
        "lc_encode_gemm_fused": (s, [_vp, _vp, f, _V, _V, f, _V, C.POINTER(lc_epilogue)]),
        "lc_encode_materialize": (s, [_vp, _vp, _V, _V]),
        "lc_materialize": (s, [_vp, _V, _V]),
        "lc_encode_conjugate": (s, [_vp, _vp, _V, _V]),
        "lc_encode_adjoint": (s, [_vp, _vp, _V, _V]),
        "lc_encode_pack": (s, [_vp, _vp, _V, _V]),
        "lc_pack": (s, [_vp, _V, _V]),
        "lc_encode_concat": (s, [_vp, _vp, _V, C.c_int32, C.c_int32, _V]),
        "lc_encode_argmax": (s, [_vp, _vp, _V, _V]),
        "lc_argmax": (s, [_vp, _V, _V]),
        "lc_encode_argmax_rows": (s, [_vp, _vp, _V, _V]),
        "lc_encode_argmax_complex": (s, [_vp, _vp, _V, C.c_int32, _V]),
        "lc_encode_sqrt": (s, [_vp, _vp, _V, _V]),
        "lc_sqrt": (s, [_vp, _V, _V]),
        "lc_encode_reciprocal": (s, [_vp, _vp, _V, _V]),
        "lc_reciprocal": (s, [_vp, _V, _V]),
        "lc_backend_gemm": (s, [_vp, _vp, _V, _V, _V, f, f]),
        "lc_add_bias": (s, [_vp, _vp, _V, _V, _V]),
        "lc_bias_grad": (s, [_vp, _vp, _V, _V]),
        "lc_mse_grad": (s, [_vp, _vp, _V, _V, _V, C.POINTER(C.c_float)]),
        "lc_sgd_step": (s, [_vp, _vp, _V, _V, f]),
        "lc_convert": (s, [_vp, _vp, _V, _V]),
        "lc_gelu": (s, [_vp, _vp, _V, _V]),
        "lc_gelu_backward": (s, [_vp, _vp, _V, _V, _V]),
        "lc_relu": (s, [_vp, _vp, _V, _V]),
        "lc_relu_backward": (s, [_vp, _vp, _V, _V, _V]),
        "lc_local_order": (s, [C.c_uint64, C.c_uint64, C.c_uint64, C.POINTER(C.c_int64), C.c_uint64,
                               C.POINTER(C.c_uint64)]),
        "lc_contiguous_placement": (s, [C.c_uint64, C.c_uint64, C.POINTER(C.c_uint64)]),
        "lc_wire_write_header": (s, [C.c_int32, C.POINTER(C.c_uint64), C.c_uint32, C.POINTER(C.c_uint8),
                                     C.POINTER(C.c_uint64)]),
        "lc_wire_parse_header": (s, [C.POINTER(C.c_uint8), C.c_uint64, C.POINTER(C.c_int32), C.POINTER(C.c_uint64),
                                     C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)]),
        "lc_pipeline_unique_id": (s, [C.POINTER(C.c_uint8)]),
        "lc_pipeline_create": (s, [C.POINTER(lc_pipeline_config), C.POINTER(C.c_uint8), C.c_int32, C.c_int32,
                                   C.c_int32, C.POINTER(_vp)]),
        "lc_pipeline_destroy": (s, [_vp]),
        "lc_pipeline_local_layers": (s, [_vp, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
        "lc_pipeline_set_weight": (s, [_vp, C.c_uint64, _vp]),
        "lc_pipeline_get_weight": (s, [_vp, C.c_uint64, _vp]),
        "lc_pipeline_get_grad": (s, [_vp, C.c_uint64, _vp]),
        "lc_pipeline_step": (s, [_vp, _vp, _vp, C.c_int32, C.POINTER(C.c_float)]),
        "lc_pipeline_get_output": (s, [_vp, _vp]),
        "lc_pipeline_last_step_ms": (s, [_vp, C.POINTER(C.c_float)]),
        "lc_pipeline_set_trace": (s, [_vp, C.c_int32]),
        "lc_pipeline_trace": (s, [_vp, _vp, C.c_uint64, C.POINTER(C.c_uint64)]),
        "lc_pipeline_init_weights": (s, [_vp, C.c_uint64, C.c_float]),
        "lc_pipeline_stream": (_vp, [_vp]),
        "lc_pipeline_debug_launches": (C.c_uint64, [_vp]),
    }
    for name, (res, args) in table.items():
        fn = getattr(L, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args


def library_path() -> Path:
    return LIB_PATH


def load() -> C.CDLL:
    """Loads the CUDA library.  Raises if it is not built: there is no fallback."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `make -C {HERE.parent}` (nvcc, sm_100a)")
        _lib = C.CDLL(str(LIB_PATH), mode=C.RTLD_GLOBAL)
        _sig(_lib)
    return _lib


def check(code: int):
    if code != OK:
        msg = load().lc_last_error().decode(errors="replace")
        raise _ERRORS.get(code, LinalgError)(code, msg)


# ---------------------------------------------------------------------------------------------
# views over torch tensors
# ---------------------------------------------------------------------------------------------

def _dtype_code(t) -> int:
    import torch
    m = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int32: I32,
         torch.complex64: C32, torch.float64: F64, torch.complex128: C64}
    if hasattr(torch, "uint32"):
        m[torch.uint32] = U32
    if hasattr(torch, "uint16"):
        m[torch.uint16] = U16
    if t.dtype not in m:
        raise TypeError(f"unsupported element type {t.dtype}")
    return m[t.dtype]


class View:
    """A strided window into a device buffer: src/abi.rs `TensorView` (buffer base, offset,
    shape, strides in elements).  ``owner`` keeps the torch storage alive."""

    __slots__ = ("c", "owner")

    def __init__(self, c: lc_view, owner):
        self.c = c
        self.owner = owner

    @staticmethod
    def of(t, dtype: int | None = None) -> "View":
        st = t.untyped_storage()
        v = lc_view()
        v.data = st.data_ptr()
        v.buffer_bytes = st.nbytes()
        v.offset = t.storage_offset()
        v.dtype = _dtype_code(t) if dtype is None else dtype
        v.rank = t.dim()
        if v.rank > MAX_RANK:
            raise InvalidArgument(ERR_INVALID_ARGUMENT, "rank above 8")
        for i, (n, s) in enumerate(zip(t.shape, t.stride())):
            if s < 0:
                raise InvalidArgument(ERR_INVALID_ARGUMENT, "negative stride")
            v.shape[i] = n
            v.strides[i] = s
        return View(v, t)

    @staticmethod
    def raw(owner, offset: int, shape, strides, dtype: int | None = None) -> "View":
        """A view with explicit metadata over ``owner``'s storage (no validation here)."""
        v = View.of(owner, dtype)
        v.c.offset = offset
        v.c.rank = len(shape)
        for i in range(MAX_RANK):
            v.c.shape[i] = shape[i] if i < len(shape) else 0
            v.c.strides[i] = strides[i] if i < len(strides) else 0
        return v

    @property
    def shape(self):
        return [self.c.shape[i] for i in range(self.c.rank)]

    @property
    def strides(self):
        return [self.c.strides[i] for i in range(self.c.rank)]

    @property
    def offset(self):
        return self.c.offset

    def ref(self):
        return C.byref(self.c)


def as_view(x) -> View:
    return x if isinstance(x, View) else View.of(x)


class Context:
    """One CUDA device and its stream (src/abi.rs `MetalContext`)."""

    def __init__(self, device: int = 0):
        L = load()
        h = _vp()
        check(L.lc_context_create(device, C.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            load().lc_context_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self):
        return load().lc_context_stream(self.h)

    def sync(self, stream=None):
        check(load().lc_sync(self.h, stream))

    def debug_wait_probe(self, limit_us: int, stream=None):
        """Enqueue a kernel whose bounded wait can only run out (failure-detection test)."""
        check(load().lc_debug_wait_probe(self.h, stream, limit_us))

    def debug_launches(self) -> list[str]:
        L = load()
        n = L.lc_debug_launches(self.h)
        out = []
        for i in range(max(0, n - 4096), n):
            s = L.lc_debug_launch_name(self.h, i)
            out.append(s.decode() if s else "?")
        return out


_default_ctx = None


def context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context(0)
    return _default_ctx


def _stream(stream):
    if stream is None:
        return None
    if hasattr(stream, "cuda_stream"):
        return stream.cuda_stream
    return stream


# ---------------------------------------------------------------------------------------------
# op API (src/ops/*.rs)
# ---------------------------------------------------------------------------------------------

def encode_contract(ctx: Context, stream, alpha, a, b, beta, c):
    """``a``, ``b``, ``c`` are (tensor_or_view, labels) pairs (src/ops/contraction.rs:1036)."""
    (av, al), (bv, bl), (cv, cl) = a, b, c
    av, bv, cv = as_view(av), as_view(bv), as_view(cv)
    check(load().lc_encode_contract(ctx.h, _stream(stream), float(alpha), av.ref(), al.encode(), bv.ref(),
                                    bl.encode(), float(beta), cv.ref(), cl.encode()))


def contract(ctx: Context, alpha, a, b, beta, c):
    (av, al), (bv, bl), (cv, cl) = a, b, c
    av, bv, cv = as_view(av), as_view(bv), as_view(cv)
    check(load().lc_contract(ctx.h, float(alpha), av.ref(), al.encode(), bv.ref(), bl.encode(), float(beta),
                             cv.ref(), cl.encode()))


def plan_contract(ctx: Context, alpha, a, b, beta, c) -> dict:
    (av, al), (bv, bl), (cv, cl) = a, b, c
    av, bv, cv = as_view(av), as_view(bv), as_view(cv)
    p = lc_contract_plan()
    check(load().lc_plan_contract(ctx.h if ctx is not None else None, float(alpha), av.ref(), al.encode(), bv.ref(), bl.encode(), float(beta),
                                  cv.ref(), cl.encode(), C.byref(p)))
    kinds = {0: "Empty", 1: "Fill", 2: "Tiled", 3: "Split", 4: "Staged", 5: "General"}
    return {"kind": kinds[p.kind], "splits": p.splits, "batch": p.batch, "m": p.m, "n": p.n, "k": p.k,
            "swap_ab": bool(p.swap_ab), "a_major": "MN" if p.a_major else "K", "b_major": "MN" if p.b_major else "K"}


def encode_gemm(ctx: Context, stream, alpha, a, b, beta, c):
    a, b, c = as_view(a), as_view(b), as_view(c)
    check(load().lc_encode_gemm(ctx.h, _stream(stream), float(alpha), a.ref(), b.ref(), float(beta), c.ref()))


def encode_gemm_noalloc(ctx: Context, stream, alpha, a, b, beta, c):
    """encode_gemm with its split-K scratch in fixed per-device arrays (no device allocation).
    Calls that may run concurrently race on those arrays; the first call on a device does set-up."""
    a, b, c = as_view(a), as_view(b), as_view(c)
    check(load().lc_encode_gemm_noalloc(ctx.h, _stream(stream), float(alpha), a.ref(), b.ref(), float(beta), c.ref()))


def encode_gemm_fused(ctx: Context, stream, alpha, a, b, beta, c, kind: int, aux=None, aux2=None, lr=0.0,
                      tile_n=0, splits=0, swap=0):
    """encode_gemm with a fused epilogue (EPI_RELU, EPI_RELU_MASK with `aux` the bf16 mask source,
    EPI_SGD with C the f32 master weights and `aux2` their bf16 copy); tile_n / splits / swap pin
    the plan (0 = the planner's choice)."""
    a, b, c = as_view(a), as_view(b), as_view(c)
    xv = as_view(aux) if aux is not None else None
    yv = as_view(aux2) if aux2 is not None else None
    e = lc_epilogue(int(kind), C.addressof(xv.c) if xv is not None else None,
                    C.addressof(yv.c) if yv is not None else None, float(lr), int(tile_n), int(splits), int(swap))
    check(load().lc_encode_gemm_fused(ctx.h, _stream(stream), float(alpha), a.ref(), b.ref(), float(beta), c.ref(),
                                      C.byref(e)))


def gemm(ctx: Context, alpha, a, b, beta, c):
    a, b, c = as_view(a), as_view(b), as_view(c)
    check(load().lc_gemm(ctx.h, float(alpha), a.ref(), b.ref(), float(beta), c.ref()))


def permute_view(view, perm) -> View:
    v = as_view(view)
    arr = (C.c_int32 * max(len(perm), 1))(*perm)
    out = lc_view()
    check(load().lc_permute_view(v.ref(), arr, len(perm), C.byref(out)))
    return View(out, v.owner)


def slice(view, ranges) -> View:  # noqa: A001 - mirrors the reference's `slice`
    v = as_view(view)
    n = len(ranges)
    starts = (C.c_uint64 * max(n, 1))(*[r.start for r in ranges])
    ends = (C.c_uint64 * max(n, 1))(*[r.stop for r in ranges])
    out = lc_view()
    check(load().lc_slice(v.ref(), starts, ends, n, C.byref(out)))
    return View(out, v.owner)


def _binary(name, ctx, stream, src, dst):
    s, d = as_view(src), as_view(dst)
    check(getattr(load(), name)(ctx.h, _stream(stream), s.ref(), d.ref()))


def encode_materialize(ctx, stream, src, dst): _binary("lc_encode_materialize", ctx, stream, src, dst)
def encode_conjugate(ctx, stream, src, dst): _binary("lc_encode_conjugate", ctx, stream, src, dst)
def encode_adjoint(ctx, stream, src, dst): _binary("lc_encode_adjoint", ctx, stream, src, dst)
def encode_pack(ctx, stream, src, dst): _binary("lc_encode_pack", ctx, stream, src, dst)
def encode_sqrt(ctx, stream, src, dst): _binary("lc_encode_sqrt", ctx, stream, src, dst)
def encode_reciprocal(ctx, stream, src, dst): _binary("lc_encode_reciprocal", ctx, stream, src, dst)
def encode_argmax(ctx, stream, x, out): _binary("lc_encode_argmax", ctx, stream, x, out)
def encode_argmax_rows(ctx, stream, x, out): _binary("lc_encode_argmax_rows", ctx, stream, x, out)


def _sync_after(fn):
    def wrapped(ctx, *args):
        fn(ctx, None, *args)
        ctx.sync()
    wrapped.__name__ = fn.__name__.replace("encode_", "")
    return wrapped


materialize = _sync_after(encode_materialize)
conjugate = _sync_after(encode_conjugate)
adjoint = _sync_after(encode_adjoint)
pack = _sync_after(encode_pack)
sqrt = _sync_after(encode_sqrt)
reciprocal = _sync_after(encode_reciprocal)
argmax = _sync_after(encode_argmax)
argmax_rows = _sync_after(encode_argmax_rows)


def encode_argmax_complex(ctx, stream, x, magnitude: str, out):
    x, o = as_view(x), as_view(out)
    check(load().lc_encode_argmax_complex(ctx.h, _stream(stream), x.ref(), {"L1": 0, "Hypot": 1}[magnitude],
                                          o.ref()))


def argmax_complex(ctx, x, magnitude: str, out):
    encode_argmax_complex(ctx, None, x, magnitude, out)
    ctx.sync()


def encode_concat(ctx, stream, parts, axis: int, dst):
    vs = [as_view(p) for p in parts]
    arr = (lc_view * max(len(vs), 1))(*[v.c for v in vs])
    d = as_view(dst)
    check(load().lc_encode_concat(ctx.h, _stream(stream), arr, len(vs), axis, d.ref()))


def concat(ctx, parts, axis: int, dst):
    encode_concat(ctx, None, parts, axis, dst)
    ctx.sync()


# ---------------------------------------------------------------------------------------------
# Backend training ops (crates/core/src/lib.rs:143-236)
# ---------------------------------------------------------------------------------------------

def backend_gemm(ctx, a, b, c, alpha, beta, stream=None):
    a, b, c = as_view(a), as_view(b), as_view(c)
    check(load().lc_backend_gemm(ctx.h, _stream(stream), a.ref(), b.ref(), c.ref(), float(alpha), float(beta)))


def add_bias(ctx, x, b, y, stream=None):
    check(load().lc_add_bias(ctx.h, _stream(stream), as_view(x).ref(), as_view(b).ref(), as_view(y).ref()))


def bias_grad(ctx, dpre, db, stream=None):
    check(load().lc_bias_grad(ctx.h, _stream(stream), as_view(dpre).ref(), as_view(db).ref()))


def mse_grad(ctx, y, target, dy, stream=None) -> float:
    loss = C.c_float(0)
    check(load().lc_mse_grad(ctx.h, _stream(stream), as_view(y).ref(), as_view(target).ref(), as_view(dy).ref(),
                             C.byref(loss)))
    return loss.value


def sgd_step(ctx, w, dw, lr, stream=None):
    check(load().lc_sgd_step(ctx.h, _stream(stream), as_view(w).ref(), as_view(dw).ref(), float(lr)))


def convert(ctx, x, y, stream=None):
    check(load().lc_convert(ctx.h, _stream(stream), as_view(x).ref(), as_view(y).ref()))


def gelu(ctx, x, y, stream=None):
    check(load().lc_gelu(ctx.h, _stream(stream), as_view(x).ref(), as_view(y).ref()))


def relu(ctx, x, y, stream=None):
    check(load().lc_relu(ctx.h, _stream(stream), as_view(x).ref(), as_view(y).ref()))


def gelu_backward(ctx, pre, dy, dx, stream=None):
    check(load().lc_gelu_backward(ctx.h, _stream(stream), as_view(pre).ref(), as_view(dy).ref(), as_view(dx).ref()))


def relu_backward(ctx, pre, dy, dx, stream=None):
    check(load().lc_relu_backward(ctx.h, _stream(stream), as_view(pre).ref(), as_view(dy).ref(), as_view(dx).ref()))


# ---------------------------------------------------------------------------------------------
# schedule / placement / wire (host only; no device needed)
# ---------------------------------------------------------------------------------------------

def local_order(stages: int, rank: int, microbatches: int):
    cap = max(2 * microbatches, 1) if microbatches <= 0xFFFFFFFF else 1
    buf = (C.c_int64 * cap)()
    n = C.c_uint64(0)
    check(load().lc_local_order(stages, rank, microbatches, buf, cap, C.byref(n)))
    return [("F", v - 1) if v > 0 else ("B", -v - 1) for v in buf[: n.value]]


def contiguous_placement(layers: int, stages: int):
    buf = (C.c_uint64 * max(layers, 1))()
    check(load().lc_contiguous_placement(layers, stages, buf))
    return list(buf[:layers])


def wire_header(dtype: int, shape) -> bytes:
    sh = (C.c_uint64 * max(len(shape), 1))(*shape)
    out = (C.c_uint8 * 48)()
    n = C.c_uint64(0)
    check(load().lc_wire_write_header(dtype, sh, len(shape), out, C.byref(n)))
    return bytes(out[: n.value])


def wire_parse(msg: bytes):
    buf = (C.c_uint8 * max(len(msg), 1)).from_buffer_copy(msg if msg else b"\0")
    dt = C.c_int32(0)
    shape = (C.c_uint64 * 8)()
    nd = C.c_uint32(0)
    off = C.c_uint64(0)
    check(load().lc_wire_parse_header(buf, len(msg), C.byref(dt), shape, C.byref(nd), C.byref(off)))
    return dt.value, list(shape[: nd.value]), off.value
