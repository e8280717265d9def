"""Shared fixtures. ``gpu``-marked tests need a CUDA device (an sm_100 B200) and the built library."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100) and libsisa_b200.so")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _no_tf32():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return torch.load(GOLDEN / f"{name}.pt", weights_only=False)
    return load


@pytest.fixture(scope="session")
def cuda_dev():
    from sisa_b200 import backends

    ok, why = backends.cuda_status(0)
    if not ok:
        pytest.fail(f"sisa_b200 cuda kernels unavailable on this GPU box: {why}")
    return torch.device("cuda", 0)


os.environ.setdefault("CUDA_MODULE_LOADING", "LAZY")
