"""Test configuration: paths and the ``gpu`` marker.

``-m "not gpu"`` runs the oracle/host/ABI tests on a CPU-only machine;
``-m gpu`` runs the parity tests on a B200.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "cutlass-complex-conv_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _library_switches_follow_env():
    """Tests pin kernels through CCV_* environment switches, which the library
    reads once; after each test the switches are re-read, so a test that
    restored the environment leaves the library as it found it."""
    yield
    import ccv_abi
    if ccv_abi._lib is not None:
        ccv_abi._lib._sync()
