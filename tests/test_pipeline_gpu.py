"""GPU parity of the 1F1B pipeline against the CPU oracle (one stage on one GPU here; the
multi-GPU runs use tests/test_pipeline_multigpu.py under several GPUs)."""
import json
from pathlib import Path

import numpy as np
import pytest

import linalg_b200 as lb
from linalg_b200 import data
from linalg_b200.pipeline import Pipeline
from oracle import oracle as O

pytestmark = pytest.mark.gpu

G = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())


def fixture():
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
    return fx, widths, ws


@pytest.mark.parametrize("act", ["gelu", "relu"])
def test_reference_mode_tiny_fixture(gpu, act):
    """crates/pipeline/tests/pipeline.rs fixture: y and dW of `train` on one stage."""
    fx, widths, ws = fixture()
    b = fx["batch"]
    xs = np.stack([np.float32(fx["x0"]), np.float32(fx["x1"])]).reshape(2 * b, widths[0])
    dys = np.stack([np.float32(fx["dy0"]), np.float32(fx["dy1"])]).reshape(2 * b, widths[-1])
    p = Pipeline(3, 0, b, 2, activation=act, dtype="f32", lr=0.0, loss="dy", widths=widths)
    for l, w in enumerate(ws):
        p.set_weight(l, w)
    p.step(xs, dys)
    y = p.output()
    ry, rdw = O.train_reference(act, widths, b, ws, [xs[:b], xs[b:]], [dys[:b], dys[b:]])
    assert np.abs(y - ry.reshape(y.shape)).max() <= 1e-5
    for l in range(3):
        assert np.abs(p.get_grad(l) - rdw[l]).max() <= 1e-5 * max(1.0, np.abs(rdw[l]).max())
    p.close()


def test_reference_mode_wider_layers(gpu):
    widths = [96, 160, 64, 128]
    b, mbs = 8, 4
    ws = [data.normal(10 + l, (widths[l], widths[l + 1]), scale=widths[l] ** -0.5) for l in range(3)]
    xs = data.normal(1, (mbs * b, widths[0]))
    dys = data.normal(2, (mbs * b, widths[-1]))
    p = Pipeline(3, 0, b, mbs, activation="gelu", dtype="f32", lr=0.0, loss="dy", widths=widths)
    for l, w in enumerate(ws):
        p.set_weight(l, w)
    p.step(xs, dys)
    ry, rdw = O.train_reference("gelu", widths, b, ws, np.split(xs, mbs), np.split(dys, mbs))
    y = p.output()
    assert np.abs(y - ry.reshape(y.shape)).max() <= 1e-5 * np.abs(ry).max()
    for l in range(3):
        g = p.get_grad(l)
        assert np.abs(g - rdw[l]).max() <= 1e-5 * np.abs(rdw[l]).max(), l
    p.close()


def test_training_step_matches_oracle_reduced_config(gpu):
    """The benchmark step on a reduced config (d=256, L=4, 8 microbatches of 16): loss within
    1e-2 relative of the CPU oracle, and the updated master weights close to the oracle's."""
    L, d, mbs, mb, lr = 4, 256, 8, 16, 1e-1
    B = mbs * mb
    master = np.stack([data.normal(100 + l, (d, d), scale=d ** -0.5) for l in range(L)])
    x = data.normal(1, (B, d))
    t = data.normal(2, (B, d))
    p = Pipeline(L, d, mb, mbs, lr=lr)
    for l in range(L):
        p.set_weight(l, master[l])
    ref = master.copy()
    losses, ref_losses = [], []
    for step in range(3):
        losses.append(p.step(x, t))
        ref_losses.append(O.mlp_step(ref, x, t, mb, lr, threads=8))
    for got, want in zip(losses, ref_losses):
        assert abs(got - want) <= 1e-2 * abs(want), (losses, ref_losses)
    assert losses[-1] < losses[0]
    for l in range(L):
        w = p.get_weight(l)
        # the update itself (W after - W before) agrees within 5% of its size
        assert np.abs(w - ref[l]).max() <= 5e-2 * np.abs(ref[l] - master[l]).max() + 1e-7
    p.close()


def test_training_step_is_deterministic(gpu):
    L, d, mbs, mb = 2, 512, 4, 64
    outs = []
    for _ in range(2):
        p = Pipeline(L, d, mb, mbs, lr=1e-3)
        p.init_weights(7, d ** -0.5)
        x = data.normal(1, (mbs * mb, d))
        t = data.normal(2, (mbs * mb, d))
        loss = p.step(x, t)
        outs.append((loss, p.get_weight(0).tobytes(), p.get_weight(1).tobytes()))
        p.close()
    assert outs[0] == outs[1]


def test_layer_chains_equal_one_launch_per_layer(gpu, tmp_path):
    """Each microbatch's layer loop runs as one chain launch (CTAs resident across layers);
    the products and their order of summation are those of one launch per layer, so the
    losses and weights match bit for bit (LC_GEMM_CHAIN=0 forces one launch per layer).  One
    microbatch per product (LC_PIPE_FUSE=1), as every stage of a multi-GPU run computes them:
    one-stage microbatch groups run as one launch per layer, not as chains."""
    import os
    import subprocess
    import sys
    here = Path(__file__).resolve().parent
    cfg = {"layers": 6, "width": 1024, "microbatch": 64, "microbatches": 4, "lr": 1e-2, "steps": 2, "seed": 5,
           "rank": 0, "world": 1, "uid": ""}
    outs = {}
    for mode in ("chain", "layers"):
        env = dict(os.environ, LC_PIPE_FUSE="1")
        if mode == "layers":
            env["LC_GEMM_CHAIN"] = "0"
        c = dict(cfg, out=str(tmp_path / f"{mode}.npz"))
        r = subprocess.run([sys.executable, str(here / "_pipeline_rank.py"), json.dumps(c)], env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        outs[mode] = np.load(tmp_path / f"{mode}.npz")
    a, b = outs["chain"], outs["layers"]
    assert a["losses"].tobytes() == b["losses"].tobytes()
    assert a["losses"][1] < a["losses"][0]
    for l in range(cfg["layers"]):
        assert a[f"w{l}"].tobytes() == b[f"w{l}"].tobytes(), l


def test_weight_update_on_two_sm_tiles(gpu, tmp_path):
    """At width 2304 the weight-gradient product has a 256 x 256 tile for every pair of SMs and
    runs on CTA pairs with cta_group::2 MMAs and the fused SGD; the update must match the one-SM
    kernel's (LC_GEMM_2SM=0) to within the rounding of a differently ordered f32 accumulation."""
    import os
    import subprocess
    import sys
    here = Path(__file__).resolve().parent
    cfg = {"layers": 2, "width": 2304, "microbatch": 64, "microbatches": 2, "lr": 1e-1, "steps": 1, "seed": 9,
           "rank": 0, "world": 1, "uid": ""}
    outs = {}
    for mode in ("two_sm", "one_sm"):
        env = dict(os.environ)
        if mode == "one_sm":
            env["LC_GEMM_2SM"] = "0"
        c = dict(cfg, out=str(tmp_path / f"{mode}.npz"))
        r = subprocess.run([sys.executable, str(here / "_pipeline_rank.py"), json.dumps(c)], env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        outs[mode] = np.load(tmp_path / f"{mode}.npz")
    a, b = outs["two_sm"], outs["one_sm"]
    assert a["losses"].tobytes() == b["losses"].tobytes()  # the forward precedes any update
    for l in range(cfg["layers"]):
        step = np.abs(a[f"w{l}"] - a[f"w0_{l}"]).max()
        assert step > 0
        assert np.abs(a[f"w{l}"] - b[f"w{l}"]).max() <= 1e-3 * step, l


@pytest.mark.parametrize("width", [1024, 8192])
def test_grouped_microbatches_equal_one_at_a_time(gpu, tmp_path, width):
    """On one stage, consecutive microbatches run as one product per layer (four by default,
    two with LC_PIPE_FUSE=2), so one pass over each weight matrix serves the group.  Each group
    product keeps the one-microbatch product's split count and orientation, so the losses and
    the updated weights equal those of one microbatch at a time (LC_PIPE_FUSE=1) bit for bit.
    Width 1024 runs the products split-K; width 8192 on CTA pairs."""
    import os
    import subprocess
    import sys
    here = Path(__file__).resolve().parent
    cfg = {"layers": 3 if width == 1024 else 2, "width": width, "microbatch": 64, "microbatches": 8, "lr": 1e-2,
           "steps": 2, "seed": 11, "rank": 0, "world": 1, "uid": ""}
    outs = {}
    for fuse in ("1", "2", "4"):
        env = dict(os.environ, LC_PIPE_FUSE=fuse)
        c = dict(cfg, out=str(tmp_path / f"f{fuse}.npz"))
        r = subprocess.run([sys.executable, str(here / "_pipeline_rank.py"), json.dumps(c)], env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        outs[fuse] = np.load(tmp_path / f"f{fuse}.npz")
    one = outs["1"]
    assert one["losses"][1] < one["losses"][0]
    for fuse in ("2", "4"):
        got = outs[fuse]
        assert got["losses"].tobytes() == one["losses"].tobytes(), fuse
        for l in range(cfg["layers"]):
            assert got[f"w{l}"].tobytes() == one[f"w{l}"].tobytes(), (fuse, l)
