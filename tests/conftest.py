"""Shared pytest configuration: the `gpu` marker and common fixtures."""

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


@pytest.fixture(scope="session")
def cuda_op():
    """The CUDA operator; GPU tests fail (not skip) if the native library is missing."""
    import torch

    from jasnamacos_b200.deform_conv import CudaDeformConv

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    return CudaDeformConv()


@pytest.fixture(scope="session")
def host_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
