import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")


def golden(name):
    """Load a golden fixture generated from the reference (tests/golden/make_golden.py)."""
    d = np.load(GOLDEN / f"{name}.npz")
    return {k: torch.from_numpy(d[k]) for k in d.files}


def rel_err(a, b):
    """max|a-b| / max|b| per tensor (the tolerance measure used throughout)."""
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    den = b.abs().max().item()
    num = (a - b).abs().max().item()
    return num / den if den > 0 else num


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from affmae_b200 import build
    build.build()
    return torch.device("cuda:0")
