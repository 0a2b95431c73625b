"""Shared pytest set-up: the `gpu` marker, import paths and CUDA fixtures."""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PACKAGE_DIR = os.path.join(ROOT, "hpc-ops-sm120_b200")
for path in (ROOT, PACKAGE_DIR, os.path.join(ROOT, "tests")):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    # Keep the file that exercises the allocation-free entry point last.
    items.sort(key=lambda item: os.path.basename(str(item.fspath)).startswith("test_zz_"))


@pytest.fixture(scope="session")
def cuda_device():
    """The B200 under test.  Reference equivalent: tests/test_attention_decode.py:36-42,
    with the capability gate moved from (12, 0) to (10, x)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA is unavailable; run the gpu tests on a B200")
    if torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("these kernel tests require an sm_100 GPU (compute capability 10.x)")
    return torch.device("cuda", torch.cuda.current_device())


@pytest.fixture(scope="module")
def device(cuda_device):
    return cuda_device
