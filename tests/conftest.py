"""Shared pytest configuration.

``-m "not gpu"`` runs the oracle and host-logic tests on any machine;
``-m gpu`` runs the CUDA parity tests, which call the C ABI of
libnvfp4_moe_cuda.so on an sm_100a device.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "x2-nvfp4-lab_b200"
for p in (ROOT, PKG_ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    """The MoE-bank path's tests run first, then the dense NVFP4 linear's
    (tests/test_linear.py, outside the bank path), so that a run with -x
    reports the bank path in full whatever the linear's tests do; the
    allocation-free entry point's test (tests/test_zz_no_alloc.py) runs after
    every other test."""
    def key(item):
        name = Path(str(item.fspath)).name
        return (name == "test_zz_no_alloc.py", name == "test_linear.py")

    items.sort(key=key)


@pytest.fixture(scope="session")
def cuda_runtime():
    """One Runtime per test session (GPU tests only). Fails loudly if the
    library or the device is missing -- there is no fallback."""
    import torch

    from vllm_nvfp4_cuda.runtime import Runtime

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.init()
    rt = Runtime()
    yield rt
    rt.synchronize()
