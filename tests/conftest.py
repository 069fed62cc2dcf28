import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_PARENT = ROOT / "pipeline-parallelism-deep-learning-library_b200"
for p in (str(ROOT), str(PKG_PARENT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def gpu():
    """The CUDA library bound to cuda:0.  GPU tests fail (not skip) when it cannot load."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a CUDA device")
    import linalg_b200 as lb

    lb.load()
    return lb
