"""Shared test setup: repo root on sys.path, the `gpu` and `slow` markers, and
the one device probe every GPU test gates on."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); runs the CUDA path")
    config.addinivalue_line("markers", "slow: long-running; excluded from the quick edit loop")


def _has_cuda() -> bool:
    if os.environ.get("KVQ_FORCE_NO_GPU") == "1":
        return False
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_CUDA = _has_cuda()


@pytest.fixture(scope="session")
def native():
    """The loaded C-ABI library. On a GPU machine a missing or unloadable
    library is a failure, never a skip: the CUDA path is the product."""
    if not HAS_CUDA:
        pytest.skip("no CUDA device")
    from kernelverify_b200 import _native
    return _native.lib()
