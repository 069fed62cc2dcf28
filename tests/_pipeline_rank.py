"""One rank of a pipeline run in its own process (one process per GPU, as the pipeline
requires), started by the pipeline tests.  Writes the losses and this rank's updated layers to
an .npz file."""
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "pipeline-parallelism-deep-learning-library_b200"))

import numpy as np  # noqa: E402

from linalg_b200 import data  # noqa: E402
from linalg_b200.pipeline import Pipeline  # noqa: E402


def main():
    cfg = json.loads(sys.argv[1])
    rank, world, out = cfg["rank"], cfg["world"], cfg["out"]
    uid = bytes.fromhex(cfg["uid"]) if cfg.get("uid") else None
    L, d, mb, mbs, lr, steps = cfg["layers"], cfg["width"], cfg["microbatch"], cfg["microbatches"], cfg["lr"], cfg["steps"]
    p = Pipeline(L, d, mb, mbs, lr=lr, rank=rank, world=world, device=rank, uid=uid, timeout_ms=60000)
    p.init_weights(cfg["seed"], d ** -0.5)
    w0 = {f"w0_{p.first + i}": p.get_weight(i) for i in range(p.count)}
    x = data.normal(1, (mb * mbs, d)) if rank == 0 else None
    t = data.normal(2, (mb * mbs, d)) if rank == world - 1 else None
    losses = [p.step(x, t) for _ in range(steps)]
    ws = {f"w{p.first + i}": p.get_weight(i) for i in range(p.count)}
    np.savez(out, losses=np.array(losses, dtype=np.float32), **ws, **w0)
    p.close()


if __name__ == "__main__":
    main()
