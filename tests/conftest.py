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


# An element outside the bar passes only where the reference's own fp32
# arithmetic is outside it too, and then at most this many times as far from
# the exact value as the reference's farthest evaluation (two valid fp32
# evaluations of an ill-conditioned element routinely differ by that factor).
FP32_NOISE_FACTOR = 2.0


def assert_close_grad(actual, expected, what="", ref32=None):
    """Gradient parity against `expected`, the oracle's exact value (float64
    throughout, at the fp32 inputs): |a - e| <= ATOL + RTOL |e| at every
    element.  An element outside that bar passes only with float64 evidence
    that the reference's own fp32 arithmetic is outside the bar at that element
    too, and `actual` is at most FP32_NOISE_FACTOR times as far from the exact
    value as the farthest of those evaluations.  `ref32` holds fp32 evaluations
    of the reference (an array or a list: the oracle's one-term-at-a-time sums
    in orders the reference's float atomics may take, its terms summed exactly
    or with q contracted as its CUDA build forms it, its golden autograd
    output).  Elements of thin Gaussians (q cancels) and elements whose terms
    cancel (d_rot is a difference of d_conic terms) carry that much fp32 noise
    in any evaluation; no blanket slack is given."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} vs {e.shape}"
    if a.size == 0:
        return
    err = np.abs(a - e)
    bar = ATOL + RTOL * np.abs(e)
    bad = err > bar
    refs = [] if ref32 is None else ([ref32] if isinstance(ref32, np.ndarray) else list(ref32))
    err32 = None
    if refs and bad.any():
        err32 = np.max([np.abs(np.asarray(r, dtype=np.float64) - e) for r in refs], axis=0)
        bad = bad & ~((err32 > bar) & (err <= FP32_NOISE_FACTOR * err32))
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, err - bar, -np.inf)), a.shape)
        extra = "" if err32 is None else f", fp32 reference error {err32[i]!r}"
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{a.size} outside atol={ATOL} rtol={RTOL} without fp32 evidence; "
            f"worst at {i}: got {a[i]!r} expected {e[i]!r}{extra} (max abs err {err.max():.3e})"
        )


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
