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


# The reference engine's unmodified Python tree, copied (not committed) by
# baseline/install_reference.py. Tests that drive the reference's own graph
# modules over this package's ops skip when it is absent.
REFERENCE_COPY = REPO / "baseline" / "_ref"


@pytest.fixture(scope="session")
def reference_modules():
    """The reference's ``scheduler`` and ``piecewise`` packages, importable,
    with their ``attn.*`` / ``kv_cache.*`` imports resolved to this package."""
    import importlib
    from types import SimpleNamespace

    if not (REFERENCE_COPY / "scheduler" / "decode_module.py").exists():
        pytest.skip("no copy of the reference engine in baseline/_ref "
                    "(python baseline/install_reference.py <reference tree>)")
    import custom_inference_engine_b200 as cie

    cie.install_reference_aliases()
    if str(REFERENCE_COPY) not in sys.path:
        sys.path.append(str(REFERENCE_COPY))
    names = dict(decode_module="scheduler.decode_module", mixed_module="scheduler.mixed_module",
                 graph_backend="scheduler.graph_backend", slots="scheduler.slots",
                 piecewise_utils="piecewise.utils", piecewise_backend="piecewise.backend")
    mods = {k: importlib.import_module(v) for k, v in names.items()}
    for m in mods.values():
        assert str(REFERENCE_COPY) in m.__file__, m.__file__
    return SimpleNamespace(**mods)
