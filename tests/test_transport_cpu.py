"""Host transports (crates/transport rebuilt in C++ behind the C ABI), on CPU.

The cases follow the reference's own transport tests: crates/transport/tests/transport.rs (run
here against both the loopback and the localhost TCP mesh) and tests/tcp_mesh.rs (processes
forming a mesh in any start order, the LNGM handshake and its rejections, a killed peer
surfacing as an error within about a second instead of a hang, a full queue blocking the
sender, an endpoint that drops promptly).
"""
import multiprocessing as mp
import os
import socket
import struct
import threading
import time

import pytest

import linalg_b200 as lb
from linalg_b200 import transport as T

MAKERS = {"loopback": T.loopback, "tcp": T.localhost_mesh}


def _free_ports(n):
    socks, ports = [], []
    for _ in range(n):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        socks.append(s)
        ports.append(s.getsockname()[1])
    for s in socks:
        s.close()
    return [f"127.0.0.1:{p}" for p in ports]


def _close(eps):
    for e in eps:
        e.close()


@pytest.mark.parametrize("kind", MAKERS)
def test_two_messages_preserve_order_and_raw_bytes(kind):
    eps = MAKERS[kind](2)
    eps[0].send(1, b"first")
    eps[0].send(1, bytes(range(256)) * 3)
    assert eps[1].recv(0, 2000) == b"first"
    assert eps[1].recv(0, 2000) == bytes(range(256)) * 3
    assert (eps[0].rank, eps[1].rank, eps[0].world) == (0, 1, 2)
    _close(eps)


@pytest.mark.parametrize("kind", MAKERS)
def test_empty_payload_and_parts(kind):
    eps = MAKERS[kind](2)
    eps[1].send(0, b"")
    eps[1].send_parts(0, [b"LN", b"", b"GL\xff\xfe"])
    assert eps[0].recv(1, 2000) == b""
    assert eps[0].recv(1, 2000) == b"LNGL\xff\xfe"
    _close(eps)


@pytest.mark.parametrize("kind", MAKERS)
def test_bad_rank_is_transport_error(kind):
    eps = MAKERS[kind](3)
    for bad in (0, 3, 99):
        with pytest.raises(lb.TransportError):
            eps[0].send(bad, b"x")
        with pytest.raises(lb.TransportError):
            eps[0].recv(bad, 10)
    with pytest.raises(lb.TransportError):
        MAKERS[kind](1)
    _close(eps)


@pytest.mark.parametrize("kind", MAKERS)
def test_timeout_returns_in_under_two_seconds(kind):
    eps = MAKERS[kind](2)
    t0 = time.monotonic()
    with pytest.raises(lb.TransportError):
        eps[0].recv(1, 200)
    assert time.monotonic() - t0 < 2.0
    _close(eps)


@pytest.mark.parametrize("kind", MAKERS)
def test_three_ranks_sources_never_merge(kind):
    eps = MAKERS[kind](3)
    eps[0].send(2, b"from zero")  # rank 1 idle
    assert eps[2].recv(0, 2000) == b"from zero"
    eps[1].send(2, b"one-a")
    eps[0].send(2, b"zero-a")
    eps[1].send(2, b"one-b")
    assert eps[2].recv(0, 2000) == b"zero-a"
    assert eps[2].recv(1, 2000) == b"one-a"
    assert eps[2].recv(1, 2000) == b"one-b"
    with pytest.raises(lb.TransportError):
        eps[2].recv(0, 50)
    _close(eps)


@pytest.mark.parametrize("kind", MAKERS)
def test_send_does_not_wait_for_receiver_and_threads_ping_pong(kind):
    eps = MAKERS[kind](2)
    t0 = time.monotonic()
    eps[0].send(1, b"a" * 1000)  # nobody receives yet
    assert time.monotonic() - t0 < 1.0
    assert eps[1].recv(0, 2000) == b"a" * 1000
    n = 200

    def pong():
        for i in range(n):
            m = eps[1].recv(0, 5000)
            eps[1].send(0, m + b"!")

    th = threading.Thread(target=pong)
    th.start()
    for i in range(n):
        eps[0].send(1, struct.pack("<I", i))
        assert eps[0].recv(1, 5000) == struct.pack("<I", i) + b"!"
    th.join()
    _close(eps)


def test_large_messages_keep_order_and_bytes():
    eps = T.localhost_mesh(2)
    payloads = [os.urandom(1 << 20) for _ in range(4)]

    def sender():
        for i in range(64):
            eps[0].send(1, payloads[i % 4] + struct.pack("<I", i))

    th = threading.Thread(target=sender)
    th.start()
    for i in range(64):
        m = eps[1].recv(0, 10_000)
        assert m[:-4] == payloads[i % 4] and struct.unpack("<I", m[-4:])[0] == i
    th.join()
    _close(eps)


# ---- tcp_mesh across processes ----------------------------------------------------------------

def _mesh_rank(rank, addrs, delay, q):
    try:
        time.sleep(delay)
        ep = T.tcp_mesh(rank, addrs, 20_000)
        world = len(addrs)
        for dst in range(world):
            if dst != rank:
                ep.send(dst, f"{rank}->{dst}".encode())
        got = sorted(ep.recv(src, 20_000).decode() for src in range(world) if src != rank)
        ep.close()
        q.put((rank, got))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("order", [(0, 1, 2), (2, 1, 0), (1, 2, 0)])
def test_three_processes_form_a_mesh_in_any_start_order(order):
    addrs = _free_ports(3)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_mesh_rank, args=(r, addrs, 0.3 * order.index(r), q)) for r in range(3)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(3))
    for p in procs:
        p.join(30)
    for r in range(3):
        assert res[r] == sorted(f"{s}->{r}" for s in range(3) if s != r), res


def _dying_rank(addrs, q):
    ep = T.tcp_mesh(1, addrs, 20_000)
    ep.send(0, b"last words")
    time.sleep(0.2)
    q.put("sent")
    os._exit(0)  # dies without closing anything


def test_peer_kill_surfaces_as_error_within_about_a_second():
    addrs = _free_ports(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_dying_rank, args=(addrs, q))
    p.start()
    ep = T.tcp_mesh(0, addrs, 20_000)
    assert ep.recv(1, 20_000) == b"last words"  # queued messages are still delivered
    p.join(30)
    t0 = time.monotonic()
    with pytest.raises(lb.TransportError):
        ep.recv(1, 10_000)
    assert time.monotonic() - t0 < 2.0
    with pytest.raises(lb.TransportError):
        for _ in range(100):  # a send fails once the failure is seen (queued ones may be accepted)
            ep.send(1, b"x" * 65536)
            time.sleep(0.01)
    ep.close()


def _raw_dial(addr):
    host, port = addr.split(":")
    for _ in range(400):
        try:
            return socket.create_connection((host, int(port)), timeout=5)
        except OSError:
            time.sleep(0.01)
    raise RuntimeError("could not dial")


def _mesh_in_thread(rank, addrs, timeout_ms, out):
    try:
        out.append(T.tcp_mesh(rank, addrs, timeout_ms))
    except lb.TransportError as e:
        out.append(e)


def test_rank_zero_accepts_a_raw_peer_with_the_lngm_handshake():
    addrs = _free_ports(2)
    out = []
    th = threading.Thread(target=_mesh_in_thread, args=(0, addrs, 10_000, out))
    th.start()
    s = _raw_dial(addrs[0])
    s.sendall(b"LNGM" + struct.pack("<II", 2, 1))
    assert s.recv(12, socket.MSG_WAITALL) == b"LNGM" + struct.pack("<II", 2, 0)
    th.join()
    ep = out[0]
    assert isinstance(ep, T.Endpoint)
    ep.send(1, b"hello")
    assert s.recv(8, socket.MSG_WAITALL) == struct.pack("<Q", 5)
    assert s.recv(5, socket.MSG_WAITALL) == b"hello"
    s.sendall(struct.pack("<Q", 3) + b"abc")
    assert ep.recv(1, 5000) == b"abc"
    ep.close()
    s.close()


@pytest.mark.parametrize("hello", [b"LNGX" + struct.pack("<II", 2, 1), b"LNGM" + struct.pack("<II", 3, 1),
                                   b"LNGM" + struct.pack("<II", 2, 0), b"LNGM" + struct.pack("<II", 2, 7)])
def test_bad_magic_world_or_rank_is_transport_error(hello):
    addrs = _free_ports(2)
    out = []
    th = threading.Thread(target=_mesh_in_thread, args=(0, addrs, 5_000, out))
    th.start()
    s = _raw_dial(addrs[0])
    s.sendall(hello)
    th.join()
    s.close()
    assert isinstance(out[0], lb.TransportError)


def test_bad_arguments_and_missing_peers():
    addrs = _free_ports(3)
    with pytest.raises(lb.TransportError):
        T.tcp_mesh(3, addrs, 100)
    with pytest.raises(lb.TransportError):
        T.tcp_mesh(0, addrs[:1], 100)
    with pytest.raises(lb.TransportError):
        T.tcp_mesh(0, addrs, 100, queue_depth=0)
    with pytest.raises(lb.TransportError):
        T.tcp_mesh(0, ["not an address", *addrs[1:]], 100)
    t0 = time.monotonic()
    with pytest.raises(lb.TransportError):
        T.tcp_mesh(1, addrs, 300)  # rank 0 never listens
    assert time.monotonic() - t0 < 5.0


def test_full_queue_blocks_the_sender_until_the_peer_reads():
    """depth 1 and a raw peer that reads nothing: sends return while the socket buffers take
    data, then block; once the peer reads, they finish."""
    addrs = _free_ports(2)
    out = []
    th = threading.Thread(target=_mesh_in_thread, args=(0, addrs, 10_000, out))
    th.start()
    s = _raw_dial(addrs[0])
    s.sendall(b"LNGM" + struct.pack("<II", 2, 1))
    s.recv(12, socket.MSG_WAITALL)
    th.join()
    ep = out[0]
    big = b"z" * (8 << 20)
    done = []

    def flood():
        for _ in range(6):
            ep.send(1, big)
        done.append(True)

    f = threading.Thread(target=flood)
    f.start()
    f.join(2.0)
    assert not done  # 48 MiB cannot all fit in a one-message queue plus the socket buffers
    got = 0
    while got < 6 * (len(big) + 8):
        chunk = s.recv(1 << 20)
        assert chunk
        got += len(chunk)
    f.join(10)
    assert done
    ep.close()
    s.close()
