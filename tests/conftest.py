"""Shared pytest setup: the ``gpu`` marker, import paths and GPU helpers.

``-m "not gpu"`` runs on any CPU machine (oracle vs golden vectors, the C ABI
exports, host-side logic, gloo multi-process tests).  ``-m gpu`` runs the
CUDA parity tests on a B200 and calls through the C ABI.
"""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG = os.path.join(ROOT, "gfx1150-inference_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


@pytest.fixture(scope="session")
def cuda_device():
    if not HAS_GPU:
        pytest.skip("no CUDA device")
    import torch

    torch.cuda.init()
    return 0


def gpu_count() -> int:
    if not HAS_GPU:
        return 0
    import torch

    return torch.cuda.device_count()
