"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 and run with ``pytest -m gpu``; everything
else runs on CPU (``pytest -m "not gpu"``). GPU tests are skipped only when the
machine has no NVIDIA device at all; on a GPU machine a missing or broken CUDA
library makes them fail, never silently pass.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running (full benchmark shapes)")


def has_nvidia_device() -> bool:
    return os.path.exists("/dev/nvidiactl") or os.path.exists("/dev/nvidia0")


def pytest_collection_modifyitems(config, items):
    if has_nvidia_device():
        return
    skip = pytest.mark.skip(reason="no NVIDIA device on this machine")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def backend():
    from vectorcore_b200.backend import CudaBackend

    b = CudaBackend.instance()
    assert b.available(), f"CUDA device unavailable: {b.last_error()}"
    return b


@pytest.fixture(scope="session")
def port():
    import oracle

    return oracle.port()


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")
