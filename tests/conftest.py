"""Shared pytest setup: the ``gpu`` marker and fixture loading helpers."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    """Fixture arrays as torch tensors (scalars stay numpy scalars)."""
    z = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for key in z.files:
        a = z[key]
        out[key] = torch.from_numpy(a.copy()) if a.ndim > 0 else a.item()
    return out


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
