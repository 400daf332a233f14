"""Shared pytest setup: the `gpu` marker, import paths, and GPU fixtures."""

from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "distraction-optimizedtransformerlayer_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libdotl")


@pytest.fixture(scope="session")
def kernels():
    """The loaded kernel module; fails (never skips) a gpu test without it."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    import kernel_ext

    k = kernel_ext.get_kernels()
    if k is None:
        pytest.fail(f"libdotl failed to load: {kernel_ext.load_error()}")
    return k


@pytest.fixture(autouse=True)
def _device_error_clean(request):
    """After every gpu test, the sticky device error word must be clear."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    import kernel_ext

    k = kernel_ext.get_kernels()
    if k is not None:
        torch.cuda.synchronize()
        word = k.device_error(clear=True)
        assert word == 0, f"a kernel gave up a bounded wait (device error word {word:#x})"
