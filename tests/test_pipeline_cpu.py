"""Multi-rank pipeline host logic on CPU: one process per stage, gloo transport.

Each rank follows the library's 1F1B order (lc_local_order) and layer placement
(lc_contiguous_placement), frames every boundary tensor with the LNGL wire header
(lc_wire_write_header / lc_wire_parse_header), and computes with the CPU oracle; the result must
equal the single-rank oracle bit for bit, as crates/pipeline/tests/pipeline.rs:541-562 requires of
the reference's loopback and TCP ranks.  A rank that dies must surface as an error on its peer
within the timeout, never as a hang (crates/transport/tests/tcp_mesh.rs:179-214).
"""
import datetime
import json
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
G = json.loads((ROOT / "tests" / "golden" / "reference_goldens.json").read_text())


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _fixture():
    fx = G["pipeline_fixture"]
    widths = fx["widths"]
    ws = []
    for l in range(len(widths) - 1):
        w = np.zeros((widths[l], widths[l + 1]), np.float32)
        for r in range(widths[l]):
            for c in range(widths[l + 1]):
                v = np.float32(np.float32(0.1) * np.float32(r + 1)) - np.float32(np.float32(0.05) * np.float32(c + 1))
                w[r, c] = np.float32(v + np.float32(np.float32(0.02) * np.float32(l)))
        ws.append(w)
    b = fx["batch"]
    xs = [np.float32(fx["x0"]).reshape(b, widths[0]), np.float32(fx["x1"]).reshape(b, widths[0])]
    dys = [np.float32(fx["dy0"]).reshape(b, widths[-1]), np.float32(fx["dy1"]).reshape(b, widths[-1])]
    return widths, ws, xs, dys, b


def _send(pending, arr: np.ndarray, dst: int):
    import linalg_b200 as lb

    msg = lb.wire_header(lb.F32, list(arr.shape)) + np.ascontiguousarray(arr, np.float32).tobytes()
    t = torch.frombuffer(bytearray(msg), dtype=torch.uint8)
    n = torch.tensor([t.numel()], dtype=torch.int64)
    pending.append((dist.isend(n, dst), n))
    pending.append((dist.isend(t, dst), t))


def _recv(src: int, cols: int) -> np.ndarray:
    import linalg_b200 as lb

    n = torch.zeros(1, dtype=torch.int64)
    dist.recv(n, src)
    t = torch.empty(int(n.item()), dtype=torch.uint8)
    dist.recv(t, src)
    msg = bytes(t.numpy())
    dtype, shape, off = lb.wire_parse(msg)
    assert dtype == lb.F32 and len(shape) == 2 and shape[1] == cols
    return np.frombuffer(msg[off:], dtype=np.float32).reshape(shape).copy()


def _rank_main(rank, world, port, act, q, die_rank=-1):
    try:
        sys.path.insert(0, str(ROOT))
        sys.path.insert(0, str(ROOT / "pipeline-parallelism-deep-learning-library_b200"))
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        import linalg_b200 as lb
        from oracle import oracle as O

        if rank == die_rank:
            os._exit(0)  # a stage that leaves between steps without sending anything
        widths, ws, xs, dys, b = _fixture()
        layers = len(widths) - 1
        owners = lb.contiguous_placement(layers, world)
        mine = [l for l in range(layers) if owners[l] == rank]
        mbs = len(xs)
        dw = {l: np.zeros_like(ws[l]) for l in mine}
        saved, ys, pending = {}, {}, []
        f = O.gelu if act == "gelu" else O.relu
        fb = O.gelu_backward if act == "gelu" else O.relu_backward
        for op, m in lb.local_order(world, rank, mbs):
            if op == "F":
                x = xs[m] if rank == 0 else _recv(rank - 1, widths[mine[0]])
                acts, pres = [x], []
                for l in mine:
                    pre = np.zeros((b, widths[l + 1]), np.float32)
                    O.gemm(O.DT_F32, acts[-1], ws[l], pre, 1.0, 0.0)
                    pres.append(pre)
                    acts.append(f(pre))
                saved[m] = (acts, pres)
                if rank == world - 1:
                    ys[m] = acts[-1]
                else:
                    _send(pending, acts[-1], rank + 1)
            else:
                acts, pres = saved.pop(m)
                g = dys[m] if rank == world - 1 else _recv(rank + 1, widths[mine[-1] + 1])
                for i in reversed(range(len(mine))):
                    l = mine[i]
                    dpre = fb(pres[i], g)
                    O.gemm(O.DT_F32, np.ascontiguousarray(acts[i].T), dpre, dw[l], 1.0, 1.0)
                    dx = np.zeros((b, widths[l]), np.float32)
                    O.gemm(O.DT_F32, dpre, np.ascontiguousarray(ws[l].T), dx, 1.0, 0.0)
                    g = dx
                if rank > 0:
                    _send(pending, g, rank - 1)
        for work, _ in pending:
            work.wait()
        q.put((rank, "ok", {l: dw[l].tobytes() for l in mine}, {m: y.tobytes() for m, y in ys.items()}))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which decides pass/fail
        q.put((rank, "error", repr(e), traceback.format_exc()))


def _run(world, act, die_rank=-1, join_timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, act, q, die_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    expected = world - (1 if die_rank >= 0 else 0)
    import queue as _q

    for _ in range(expected):
        try:
            rank, status, a, bb = q.get(timeout=join_timeout)
        except _q.Empty:
            break
        results[rank] = (status, a, bb)
    for p in procs:
        p.join(timeout=20)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("act", ["gelu", "relu"])
def test_multirank_gloo_bitwise_equals_single_rank(world, act):
    from oracle import oracle as O

    widths, ws, xs, dys, b = _fixture()
    ry, rdw = O.train_reference(act, widths, b, ws, xs, dys)
    res = _run(world, act)
    assert sorted(res) == list(range(world)), res
    for r, (status, dwb, yb) in res.items():
        assert status == "ok", (r, dwb, yb)
        for l, raw in dwb.items():
            assert raw == rdw[l].tobytes(), f"dW[{l}] bits differ on rank {r}"
        for m, raw in yb.items():
            assert raw == ry[m].tobytes(), f"y[{m}] bits differ"


def test_dead_peer_surfaces_as_error_not_hang():
    res = _run(2, "gelu", die_rank=1, join_timeout=60)
    assert 0 in res, "rank 0 neither finished nor reported: it hung"
    status, msg, _ = res[0]
    assert status == "error", res[0]
