"""Shared test setup: import paths, the gpu marker, seeds, golden fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "open-supersampling_b200"
for p in (ROOT, PKG, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = Path(__file__).resolve().parent / "golden"

# Tolerance of the parity bar for fp32 images and gradients: |a - b| <= ATOL + RTOL * |b|.
ATOL = 1e-5
RTOL = 1e-4


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0xC0DA)
    np.random.seed(0xC0DA)


@pytest.fixture
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def golden_case(data: dict, name: str) -> dict:
    pre = f"{name}_"
    return {k[len(pre):]: v for k, v in data.items() if k.startswith(pre)}


def assert_close_grad(actual, expected, what=""):
    """Gradient parity: the image bar plus an absolute slack of 1e-6 of the
    tensor's largest magnitude.  Gradients are fp32 sums of up to 256 x (list
    length) terms; elements that cancel to a small value (d_rot is a difference
    of d_conic terms) keep the summation noise of their large terms."""
    e = np.asarray(expected, dtype=np.float64)
    scale = float(np.abs(e).max()) if e.size else 0.0
    assert_close(actual, expected, atol=ATOL + 1e-6 * scale, rtol=RTOL, what=what)


def assert_close(actual, expected, atol=ATOL, rtol=RTOL, what=""):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} vs {e.shape}"
    if a.size == 0:
        return
    err = np.abs(a - e)
    bound = atol + rtol * np.abs(e)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), a.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{a.size} outside atol={atol} rtol={rtol}; "
            f"worst at {i}: got {a[i]!r} expected {e[i]!r} (max abs err {err.max():.3e})"
        )
