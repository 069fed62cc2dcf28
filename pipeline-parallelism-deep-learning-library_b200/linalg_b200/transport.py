"""Host transports between pipeline ranks (crates/transport's `loopback`, `localhost_mesh` and
`tcp_mesh`, behind the library's C ABI).  Messages are opaque bytes; every failure raises
``TransportError``.  ``send_tensor`` / ``recv_tensor`` move LNGL-framed device tensors, as the
reference pipeline's send_tensor / recv_tensor do."""
from __future__ import annotations

import ctypes as C

from . import as_view, check, load

_vp = C.c_void_p


def _sig(L):
    s = C.c_int32
    table = {
        "lc_transport_loopback": (s, [C.c_uint32, C.POINTER(_vp)]),
        "lc_transport_localhost_mesh": (s, [C.c_uint32, C.POINTER(_vp)]),
        "lc_transport_tcp_mesh": (s, [C.c_uint32, C.POINTER(C.c_char_p), C.c_uint32, C.c_int64, C.c_uint32,
                                      C.POINTER(_vp)]),
        "lc_transport_destroy": (s, [_vp]),
        "lc_transport_rank": (C.c_uint32, [_vp]),
        "lc_transport_world": (C.c_uint32, [_vp]),
        "lc_transport_send": (s, [_vp, C.c_uint32, C.c_char_p, C.c_uint64]),
        "lc_transport_send_parts": (s, [_vp, C.c_uint32, C.POINTER(_vp), C.POINTER(C.c_uint64), C.c_uint32]),
        "lc_transport_recv": (s, [_vp, C.c_uint32, C.c_int64, C.POINTER(C.POINTER(C.c_uint8)),
                                  C.POINTER(C.c_uint64)]),
        "lc_transport_free": (None, [C.POINTER(C.c_uint8)]),
        "lc_transport_send_tensor": (s, [_vp, C.c_uint32, _vp, _vp]),
        "lc_transport_recv_tensor": (s, [_vp, C.c_uint32, C.c_int64, _vp, _vp]),
    }
    for name, (res, args) in table.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


_L = None


def _lib():
    global _L
    if _L is None:
        _L = _sig(load())
    return _L


class Endpoint:
    """One rank's endpoint.  ``close()`` sends what is queued, then closes the connections."""

    def __init__(self, handle):
        self.h = handle

    @property
    def rank(self) -> int:
        return _lib().lc_transport_rank(self.h)

    @property
    def world(self) -> int:
        return _lib().lc_transport_world(self.h)

    def send(self, dest: int, data: bytes):
        check(_lib().lc_transport_send(self.h, dest, bytes(data), len(data)))

    def send_parts(self, dest: int, parts):
        parts = [bytes(p) for p in parts]
        bufs = [C.create_string_buffer(p, len(p)) for p in parts]
        ptrs = (_vp * max(1, len(parts)))(*[C.cast(b, _vp) for b in bufs])
        lens = (C.c_uint64 * max(1, len(parts)))(*[len(p) for p in parts])
        check(_lib().lc_transport_send_parts(self.h, dest, ptrs, lens, len(parts)))

    def recv(self, src: int, timeout_ms: int = -1) -> bytes:
        data = C.POINTER(C.c_uint8)()
        n = C.c_uint64(0)
        check(_lib().lc_transport_recv(self.h, src, int(timeout_ms), C.byref(data), C.byref(n)))
        try:
            return C.string_at(data, n.value)
        finally:
            _lib().lc_transport_free(data)

    def send_tensor(self, dest: int, ctx, t):
        v = as_view(t)
        check(_lib().lc_transport_send_tensor(self.h, dest, ctx.h, C.addressof(v.c)))

    def recv_tensor(self, src: int, ctx, t, timeout_ms: int = -1):
        v = as_view(t)
        check(_lib().lc_transport_recv_tensor(self.h, src, int(timeout_ms), ctx.h, C.addressof(v.c)))

    def close(self):
        if self.h:
            _lib().lc_transport_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _many(fn, world: int):
    hs = (_vp * max(1, world))()
    check(fn(world, hs))
    return [Endpoint(hs[i]) for i in range(world)]


def loopback(world: int) -> list[Endpoint]:
    return _many(_lib().lc_transport_loopback, world)


def localhost_mesh(world: int) -> list[Endpoint]:
    return _many(_lib().lc_transport_localhost_mesh, world)


def tcp_mesh(rank: int, addrs, connect_timeout_ms: int = 10_000, queue_depth: int = 4) -> Endpoint:
    arr = (C.c_char_p * max(1, len(addrs)))(*[a.encode() for a in addrs])
    h = _vp()
    check(_lib().lc_transport_tcp_mesh(rank, arr, len(addrs), int(connect_timeout_ms), queue_depth, C.byref(h)))
    return Endpoint(h)
