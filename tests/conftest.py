"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` tests run on any CPU host (oracle vs golden fixtures, host
logic, the C-ABI library's exports); `-m gpu` tests call the CUDA library
through its C ABI on a B200 and compare with the oracle.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO / "project-glm5x_b200", REPO / "oracle", REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) device")


def _has_b200() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_b200():
        return
    skip = pytest.mark.skip(reason="needs a B200 (sm_100) GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(REPO / "tests" / "golden" / "reference_golden.npz")
