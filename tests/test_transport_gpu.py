"""LNGL-framed device tensors over the host transports (crates/pipeline/src/lib.rs:71-98
`send_tensor` / `recv_tensor`): download, frame, send; receive, check dtype and shape, upload."""
import numpy as np
import pytest
import torch

import linalg_b200 as lb
from linalg_b200 import transport as T

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["loopback", "tcp"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_framed_tensor_round_trip(gpu, kind, dtype):
    ctx = lb.Context(0)
    eps = T.loopback(2) if kind == "loopback" else T.localhost_mesh(2)
    x = torch.randn(64, 8192, device="cuda").to(dtype)
    eps[0].send_tensor(1, ctx, x)
    y = torch.zeros_like(x)
    eps[1].recv_tensor(0, ctx, y, 10_000)
    assert torch.equal(x.view(torch.int16 if dtype != torch.float32 else torch.int32),
                       y.view(torch.int16 if dtype != torch.float32 else torch.int32))
    # the frame itself is the reference's: LNGL header + raw payload
    eps[0].send_tensor(1, ctx, x[:2, :3].contiguous())
    raw = eps[1].recv(0, 10_000)
    tag = {torch.float32: lb.F32, torch.bfloat16: lb.BF16, torch.float16: lb.F16}[dtype]
    assert raw[:len(lb.wire_header(tag, [2, 3]))] == lb.wire_header(tag, [2, 3])
    for e in eps:
        e.close()
    ctx.close()


def test_framed_tensor_rejections(gpu):
    ctx = lb.Context(0)
    eps = T.loopback(2)
    x = torch.randn(4, 6, device="cuda")
    eps[0].send_tensor(1, ctx, x)
    with pytest.raises(lb.ShapeError):
        eps[1].recv_tensor(0, ctx, torch.zeros(6, 4, device="cuda"), 1000)
    eps[0].send_tensor(1, ctx, x)
    with pytest.raises(lb.DtypeError):
        eps[1].recv_tensor(0, ctx, torch.zeros(4, 6, device="cuda", dtype=torch.bfloat16), 1000)
    eps[0].send(1, b"LNGX" + bytes(12))
    with pytest.raises(lb.WireError):
        eps[1].recv_tensor(0, ctx, torch.zeros(4, 6, device="cuda"), 1000)
    with pytest.raises(lb.ShapeError):
        eps[0].send_tensor(1, ctx, x.t())  # not row-major
    y = torch.zeros(4, 6, device="cuda")
    with pytest.raises(lb.TransportError):
        eps[1].recv_tensor(0, ctx, y, 50)  # nothing queued: times out
    assert torch.count_nonzero(y) == 0
    for e in eps:
        e.close()
    ctx.close()
