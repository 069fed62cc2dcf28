"""1F1B pipeline stage (crates/pipeline/src/lib.rs `train`, rebuilt one stage per GPU).

Each process owns one stage on one GPU.  Rank 0 creates the communicator id with
:func:`unique_id`; the caller distributes it (torch.distributed, a file, ...) and every rank
builds its :class:`Pipeline` with it.  Layers follow ``contiguous_placement``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import BF16, F32, check, lc_pipeline_config, load

ID_BYTES = 128


def unique_id() -> bytes:
    buf = (C.c_uint8 * ID_BYTES)()
    check(load().lc_pipeline_unique_id(buf))
    return bytes(buf)


class Pipeline:
    def __init__(self, layers: int, width: int, microbatch: int, microbatches: int, *, activation: str = "relu",
                 dtype: str = "bf16", lr: float = 1e-3, loss: str = "mse", rank: int = 0, world: int = 1,
                 device: int = 0, uid: bytes | None = None, widths=None, timeout_ms: int = 60000):
        L = load()
        cfg = lc_pipeline_config()
        cfg.layers = layers
        cfg.width = width
        self._widths = None
        if widths is not None:
            self._widths = (C.c_uint64 * len(widths))(*widths)
            cfg.widths = C.cast(self._widths, C.POINTER(C.c_uint64))
        cfg.microbatch = microbatch
        cfg.microbatches = microbatches
        cfg.activation = {"gelu": 0, "relu": 1}[activation]
        cfg.compute_dtype = {"bf16": BF16, "f32": F32}[dtype]
        cfg.lr = lr
        cfg.loss = {"dy": 0, "mse": 1}[loss]
        cfg.timeout_ms = timeout_ms
        self.widths = list(widths) if widths is not None else [width] * (layers + 1)
        self.rank, self.world = rank, world
        self.microbatch, self.microbatches = microbatch, microbatches
        idbuf = (C.c_uint8 * ID_BYTES).from_buffer_copy(uid) if uid is not None else None
        h = C.c_void_p()
        check(L.lc_pipeline_create(C.byref(cfg), idbuf, rank, world, device, C.byref(h)))
        self.h = h
        first, count = C.c_uint64(), C.c_uint64()
        check(L.lc_pipeline_local_layers(self.h, C.byref(first), C.byref(count)))
        self.first, self.count = first.value, count.value

    def close(self):
        if getattr(self, "h", None):
            load().lc_pipeline_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _shape(self, index):
        g = self.first + index
        return self.widths[g], self.widths[g + 1]

    def set_weight(self, index: int, w: np.ndarray):
        w = np.ascontiguousarray(w, dtype=np.float32)
        assert w.shape == self._shape(index)
        check(load().lc_pipeline_set_weight(self.h, index, w.ctypes.data))

    def init_weights(self, seed: int, stddev: float):
        check(load().lc_pipeline_init_weights(self.h, seed, stddev))

    def get_weight(self, index: int) -> np.ndarray:
        out = np.empty(self._shape(index), dtype=np.float32)
        check(load().lc_pipeline_get_weight(self.h, index, out.ctypes.data))
        return out

    def get_grad(self, index: int) -> np.ndarray:
        out = np.empty(self._shape(index), dtype=np.float32)
        check(load().lc_pipeline_get_grad(self.h, index, out.ctypes.data))
        return out

    def step(self, x=None, target=None, on_device: bool = False) -> float:
        """One training step.  ``x`` (rank 0) and ``target``/dy (last rank) are f32 [B, width]:
        numpy arrays or pinned/pageable host memory (copied inside the step), or device
        pointers / CUDA tensors with ``on_device``."""

        def ptr(a):
            if a is None:
                return None
            if hasattr(a, "data_ptr"):
                return a.data_ptr()
            a = np.ascontiguousarray(a, dtype=np.float32)
            self._keep.append(a)
            return a.ctypes.data

        self._keep = []
        loss = C.c_float(0)
        check(load().lc_pipeline_step(self.h, ptr(x), ptr(target), 1 if on_device else 0, C.byref(loss)))
        self._keep = []
        return loss.value

    def output(self) -> np.ndarray:
        out = np.empty((self.microbatches * self.microbatch, self.widths[-1]), dtype=np.float32)
        check(load().lc_pipeline_get_output(self.h, out.ctypes.data))
        return out

    @property
    def stream(self) -> int:
        return load().lc_pipeline_stream(self.h)

    def debug_launches(self) -> int:
        return load().lc_pipeline_debug_launches(self.h)

    @property
    def last_step_ms(self) -> float:
        ms = C.c_float(0)
        check(load().lc_pipeline_last_step_ms(self.h, C.byref(ms)))
        return ms.value

    def set_trace(self, on: bool = True):
        """Record CUDA events around every op of later steps (see trace())."""
        check(load().lc_pipeline_set_trace(self.h, 1 if on else 0))

    def trace(self) -> np.ndarray:
        """The last traced step: rows of (kind, first microbatch or layer, start ms, end ms), kind 1
        forward, -1 backward, 2 weight update, times from the step's start on this stage."""
        L = load()
        n = C.c_uint64(0)
        check(L.lc_pipeline_trace(self.h, None, 0, C.byref(n)))
        out = np.zeros((n.value, 4), np.float32)
        if n.value:
            check(L.lc_pipeline_trace(self.h, out.ctypes.data_as(C.c_void_p), n.value, C.byref(n)))
        return out


def trace_summary(rec: np.ndarray, step_ms: float) -> dict:
    """Busy time of a stage (the union of its ops' compute intervals, forwards, backwards and
    weight updates) against its step time; the rest is time the stage had nothing it could run:
    the 1F1B fill and drain, and waits on transfers."""
    rec = [tuple(float(v) for v in r) for r in rec]
    step_ms = float(step_ms)
    iv = sorted((a, b) for _, _, a, b in rec)
    busy, cur_a, cur_b = 0.0, None, None
    for a, b in iv:
        if cur_b is None or a > cur_b:
            if cur_b is not None:
                busy += cur_b - cur_a
            cur_a, cur_b = a, b
        else:
            cur_b = max(cur_b, b)
    if cur_b is not None:
        busy += cur_b - cur_a
    fwd = [b - a for k, _, a, b in rec if k == 1]
    bwd = [b - a for k, _, a, b in rec if k == -1]
    upd = [b - a for k, _, a, b in rec if k == 2]
    first_bwd = min([a for k, _, a, b in rec if k == -1], default=0.0)
    return {"step_ms": step_ms, "busy_ms": busy, "idle_ms": step_ms - busy,
            "forward_ms_mean": float(np.mean(fwd)) if fwd else 0.0,
            "backward_ms_mean": float(np.mean(bwd)) if bwd else 0.0,
            "update_ms_total": float(np.sum(upd)) if upd else 0.0,
            "first_backward_at_ms": first_bwd, "ops": int(len(rec))}
