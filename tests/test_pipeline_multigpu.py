"""Multi-GPU 1F1B: stages on separate GPUs, activations and gradients over NCCL send/recv.

The reference's invariant (crates/pipeline/tests/pipeline.rs:518-562): splitting the layers over
more ranks changes nothing in the result.  Every layer runs the same kernels on the same inputs
whichever stage holds it, so the losses and the updated weights must equal the one-GPU run bit
for bit.  One process per GPU (tests/_pipeline_rank.py), started fresh so that no CUDA context
is inherited; skipped where the box has fewer GPUs than ranks.
"""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from linalg_b200.pipeline import Pipeline, unique_id
from linalg_b200 import data

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent
CFG = {"layers": 4, "width": 1024, "microbatch": 32, "microbatches": 8, "lr": 1e-2, "steps": 2, "seed": 77}


def _gpus() -> int:
    # asked in a child process, so this one creates no CUDA state before the ranks start
    out = subprocess.run([sys.executable, "-c", "import torch; print(torch.cuda.device_count())"],
                         capture_output=True, text=True, timeout=300)
    return int(out.stdout.strip() or 0)


def _single_gpu_reference():
    c = CFG
    p = Pipeline(c["layers"], c["width"], c["microbatch"], c["microbatches"], lr=c["lr"])
    p.init_weights(c["seed"], c["width"] ** -0.5)
    x = data.normal(1, (c["microbatch"] * c["microbatches"], c["width"]))
    t = data.normal(2, (c["microbatch"] * c["microbatches"], c["width"]))
    losses = [p.step(x, t) for _ in range(c["steps"])]
    ws = [p.get_weight(l) for l in range(c["layers"])]
    p.close()
    return np.array(losses, dtype=np.float32), ws


@pytest.mark.parametrize("world", [2, 4])
def test_stages_over_nccl_equal_one_gpu(gpu, tmp_path, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    uid = unique_id().hex()
    procs = []
    for rank in range(world):
        cfg = dict(CFG, rank=rank, world=world, uid=uid, out=str(tmp_path / f"rank{rank}.npz"))
        procs.append(subprocess.Popen([sys.executable, str(HERE / "_pipeline_rank.py"), json.dumps(cfg)],
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    logs = []
    for pr in procs:
        try:
            out, _ = pr.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        logs.append(out)
    assert all(pr.returncode == 0 for pr in procs), "\n".join(logs)
    ref_losses, ref_ws = _single_gpu_reference()
    seen = set()
    for rank in range(world):
        z = np.load(tmp_path / f"rank{rank}.npz")
        if rank == world - 1:
            assert z["losses"].tobytes() == ref_losses.tobytes(), (z["losses"], ref_losses)
        for key in z.files:
            if key.startswith("w") and not key.startswith("w0_"):  # w0_* are the initial weights
                g = int(key[1:])
                seen.add(g)
                assert z[key].tobytes() == ref_ws[g].tobytes(), f"layer {g} differs on rank {rank}"
    assert seen == set(range(CFG["layers"]))
