"""Shared pytest setup.

Marker ``gpu``: the test needs a CUDA device (sm_100) and the built native
library.  ``python -m pytest tests -m "not gpu"`` runs everything else on CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_ROOT = ROOT / "mps-pointops_b200"
for p in (str(ROOT), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built native library")


def golden(name: str) -> dict:
    """Load tests/golden/<name>.npz as {case: {field: array}}."""
    z = np.load(GOLDEN / f"{name}.npz")
    cases: dict = {}
    for key in z.files:
        if "/" in key:
            case, field = key.split("/", 1)
            cases.setdefault(case, {})[field] = z[key]
        else:
            cases[key] = z[key]
    return cases


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device not available")
    return torch.device("cuda", 0)
