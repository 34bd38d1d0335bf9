"""Test configuration: the `gpu` marker, build-on-demand of the native
library / pack / oracle, and shared helpers."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session", autouse=True)
def native_build():
    """Builds libcutriton_b200.so, the kernel pack and the oracle if stale.
    On the GPU box the prebuilt files that travel with the tree are used;
    the rebuild is skipped when nvcc is unavailable."""
    from cutriton_b200 import _build

    if _build.NVCC.exists():
        _build.build_all()
    from oracle import ops

    ops.build()
    yield


@pytest.fixture()
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for gpu tests")
    torch.cuda.init()
    return torch.device("cuda:0")
