"""Shared pytest configuration.

Markers: ``gpu`` -- needs a CUDA (sm_100) device; everything else runs on a
CPU-only host.  The repository root is put on ``sys.path`` so ``oracle`` and
``rotalabs_accel_b200`` import without installation.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (run with -m gpu)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda_lib():
    """The built C-ABI library on a GPU host (built on demand)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rotalabs_accel_b200 import build, _capi
    build.build()
    return _capi.load_library()
