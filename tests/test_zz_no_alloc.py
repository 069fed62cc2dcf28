"""lc_encode_gemm_noalloc against lc_encode_gemm, through the C ABI.

The allocation-free entry point plans and launches exactly what lc_encode_gemm does, with its
split-K scratch in fixed per-device arrays, so its results must be bit-identical; two calls in a
row check that the first leaves nothing behind (its tile counters are zeroed before each split
launch).  Named to be collected last, and self-contained so that it also passes alone.
"""
import numpy as np
import pytest
import torch

import linalg_b200 as lb

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx(gpu):
    return lb.Context(0)


def _bits(t):
    a = t.detach().cpu().contiguous()
    return a.view(torch.int32).numpy() if a.dtype == torch.float32 else a.view(torch.int16).numpy()


def _operands(m, n, k, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(dtype).cuda()
    b = torch.randn(k, n, generator=g).to(dtype).cuda()
    c0 = torch.randn(m, n, generator=g).to(dtype).cuda()
    return a, b, c0


# (m, n, k, dtype, alpha, beta, expected plan): a 2-way split of 16-bit inputs (64 x 8192 x 8192
# bf16), which runs as a CTA pair reducing through distributed shared memory and so touches no
# scratch; the in-kernel fixup in the fixed scratch (1024^2 x 2048 f32, 2 splits, tile counters);
# the separate reduce kernel (37 splits, 9.25 MiB of partials); and a product that does not split.
CASES = [
    (64, 8192, 8192, torch.bfloat16, 1.0, 0.0, ("Split", 2)),
    (1024, 1024, 2048, torch.float32, 0.5, 0.25, ("Split", 2)),
    (256, 256, 65536, torch.float32, 1.0, -1.5, ("Split", 37)),
    (2048, 2048, 256, torch.bfloat16, 1.0, 1.0, ("Tiled", 1)),
]


@pytest.mark.parametrize("m,n,k,dtype,alpha,beta,expect", CASES)
def test_noalloc_matches_encode_gemm_twice(ctx, m, n, k, dtype, alpha, beta, expect):
    a, b, c0 = _operands(m, n, k, dtype, seed=m + n + k)
    plan = lb.plan_contract(ctx, alpha, (a, "ik"), (b, "kj"), beta, (c0, "ij"))
    assert (plan["kind"], plan["splits"]) == expect
    want = c0.clone()
    lb.encode_gemm(ctx, None, alpha, a, b, beta, want)
    got1, got2 = c0.clone(), c0.clone()
    lb.encode_gemm_noalloc(ctx, None, alpha, a, b, beta, got1)
    lb.encode_gemm_noalloc(ctx, None, alpha, a, b, beta, got2)
    ctx.sync()
    w = _bits(want)
    assert np.array_equal(_bits(got1), w)
    assert np.array_equal(_bits(got2), w)


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 2048), (256, 256, 65536)])
def test_noalloc_on_a_caller_stream(ctx, m, n, k):
    """Shapes whose split really uses the fixed arrays: the in-kernel fixup (partials and tile
    counters) and the separate reduce kernel (partials only)."""
    a, b, c0 = _operands(m, n, k, torch.float32, seed=7)
    want = c0.clone()
    lb.encode_gemm(ctx, None, 1.0, a, b, 0.5, want)
    ctx.sync()
    s = torch.cuda.Stream()
    got1, got2 = c0.clone(), c0.clone()
    torch.cuda.synchronize()
    lb.encode_gemm_noalloc(ctx, s.cuda_stream, 1.0, a, b, 0.5, got1)
    lb.encode_gemm_noalloc(ctx, s.cuda_stream, 1.0, a, b, 0.5, got2)
    s.synchronize()
    assert np.array_equal(_bits(got1), _bits(want))
    assert np.array_equal(_bits(got2), _bits(want))


_COUNTER_REFUSAL = r"""
import sys
sys.path.insert(0, sys.argv[1])
import numpy as np, torch
import linalg_b200 as lb
ctx = lb.Context(0)
g = torch.Generator(device="cpu").manual_seed(5)
a = torch.randn(2100, 1, 96, generator=g).cuda()
b = torch.randn(2100, 96, 1, generator=g).cuda()
c0 = torch.randn(2100, 1, 1, generator=g).cuda()
plan = lb.plan_contract(ctx, 1.0, (a, "bik"), (b, "bkj"), 0.0, (c0, "bij"))
assert (plan["kind"], plan["splits"]) == ("Split", 3), plan
c = c0.clone()
try:
    lb.encode_gemm_noalloc(ctx, None, 1.0, a, b, 0.0, c)
except lb.InvalidArgument as e:
    assert "tile counters" in str(e), e
else:
    raise AssertionError("2100 tiles x 4 counters passed a fixed scratch of 8192 counters")
ctx.sync()
assert torch.equal(c, c0)
print("refused")
"""


def test_noalloc_rejects_more_tile_counters_than_it_holds():
    """A 3-way split (LC_SPLITK pins it) of 2100 one-element products: 24 KiB of partials fit,
    but the fixup's 4 counters per tile (8400) do not fit the 8192 fixed counters, so the call
    is refused before any launch and C is unchanged.  In a child process, because LC_SPLITK is
    read once per process."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    pkg = Path(__file__).resolve().parents[1] / "pipeline-parallelism-deep-learning-library_b200"
    r = subprocess.run([sys.executable, "-c", _COUNTER_REFUSAL, str(pkg)], env=dict(os.environ, LC_SPLITK="3"),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "refused" in r.stdout, r.stdout + r.stderr


def test_noalloc_rejects_oversize_split(ctx):
    # 8 splits of a 2048 x 1024 f32 output need 64 MiB of partials, above the fixed 16 MiB
    a, b, c0 = _operands(2048, 1024, 16384, torch.float32, seed=3)
    plan = lb.plan_contract(ctx, 1.0, (a, "ik"), (b, "kj"), 0.0, (c0, "ij"))
    assert plan["kind"] == "Split" and plan["splits"] * 2048 * 1024 * 4 > 16 << 20
    c = c0.clone()
    with pytest.raises(lb.InvalidArgument, match="split-K partials need"):
        lb.encode_gemm_noalloc(ctx, None, 1.0, a, b, 0.0, c)
    ctx.sync()
    assert np.array_equal(_bits(c), _bits(c0))  # nothing launched


def test_noalloc_rejects_operands_that_need_staging(ctx):
    # A read with stride 2 along K and along M: no unit stride, so lc_encode_gemm would stage it
    g = torch.Generator(device="cpu").manual_seed(11)
    big = torch.randn(512, 1024, generator=g).cuda()
    a = lb.View.raw(big, 0, [256, 256], [2048, 2])
    b = torch.randn(256, 256, generator=g).cuda()
    c0 = torch.zeros(256, 256, device="cuda")
    assert lb.plan_contract(ctx, 1.0, (a, "ik"), (b, "kj"), 0.0, (c0, "ij"))["kind"] == "Staged"
    c = c0.clone()
    with pytest.raises(lb.InvalidArgument, match="staging"):
        lb.encode_gemm_noalloc(ctx, None, 1.0, a, b, 0.0, c)
    ctx.sync()
    assert np.array_equal(_bits(c), _bits(c0))
