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


# ---- attention parity bound -------------------------------------------------------
# The path's fp16 bound: attention outputs within 2e-3 RELATIVE of the reference's
# numpy path (fp16 storage, fp32 accumulate).  Applied per query row (one
# sequence's (heads, head_dim) output): max|got - ref| <= 2e-3 * max|ref|.  The
# element-wise relative error is reported too, with a floor of 1 % of the row's
# largest |ref| (outputs are softmax averages; elements far below the row's
# scale carry the absolute error of the fp32 sums, not a relative one).
FP16_REL = 2e-3


def attention_errors(got, ref):
    """(normwise, elementwise) relative errors, the worst row of each."""
    import numpy as np

    g = np.asarray(got, dtype=np.float32)
    r = np.asarray(ref, dtype=np.float32)
    g = g.reshape(-1, *g.shape[-2:]) if g.ndim >= 2 else g.reshape(1, 1, -1)
    r = r.reshape(g.shape)
    d = np.abs(g - r)
    row_max = np.abs(r).reshape(r.shape[0], -1).max(axis=1)
    row_err = d.reshape(d.shape[0], -1).max(axis=1)
    with np.errstate(divide="ignore", invalid="ignore"):
        norm = np.where(row_max > 0, row_err / row_max, np.where(row_err > 0, np.inf, 0.0))
        floor = 1e-2 * row_max[:, None, None]
        elem = d / np.maximum(np.abs(r), floor)
        elem = np.where(np.isfinite(elem), elem, np.where(d > 0, np.inf, 0.0))
    return float(norm.max()), float(elem.max())


def assert_attention_close(got, ref, what: str = "", rel: float = FP16_REL):
    """Assert the fp16 bound row by row and log the achieved errors (to the file
    named by KVC_PARITY_LOG, when set)."""
    norm, elem = attention_errors(got, ref)
    path = os.environ.get("KVC_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(f"{what}\tnormwise_rel={norm:.3e}\telementwise_rel={elem:.3e}\tbound={rel:g}\n")
    assert norm <= rel, f"{what}: max|got-ref| / max|ref| = {norm:.3e} > {rel:g}"
    return norm, elem
