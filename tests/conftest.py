"""Test configuration: the `gpu` marker, import paths, shared fixtures.

Tests marked gpu need a B200 and the built libsdb.so; the rest run on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "stable-diffusion.assembly_b200"
for p in (ROOT, PKG, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built kernel library")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import sdb

    sdb.load()
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """GPU tests must leave the device error word clear (no timeout, range or bounds bits)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    import sdb

    status = sdb.device_status(clear=True)
    assert status == 0, f"device error word 0x{status:x} after {request.node.name}"
