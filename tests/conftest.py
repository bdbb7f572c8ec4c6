"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200 for the native kernels); they
are skipped when none is present. Every other test runs on the CPU.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device and the native library")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="requires a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def native_lib():
    """Loads the native library, building it first when sources are newer."""
    from gram_newton_schulz_ampere_b200 import _native, build

    if build.is_stale() and build.nvcc_path():
        build.build()
    return _native.load()


@pytest.fixture
def cuda_device(native_lib):
    import torch

    device = torch.device("cuda", torch.cuda.current_device())
    yield device
    torch.cuda.synchronize(device)
    from gram_newton_schulz_ampere_b200 import _native

    status = _native.device_status(clear=True)
    assert status == 0, f"a kernel's bounded wait gave up (device status {status})"
