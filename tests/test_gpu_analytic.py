"""Analytic-Splatting pixel integral on the GPU (oss_b200.analytic over
csrc/analytic.cu) against the reference's own values and autograd
(tests/golden/analytic_cases.npz, made by tests/golden/make_analytic_golden.py):
values within 1e-5 abs / 1e-4 rel, gradients with respect to the offsets and the
four inverse-covariance entries within the same bar plus 1e-6 of each tensor's
largest magnitude."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import assert_close, assert_close_grad

pytestmark = pytest.mark.gpu

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "analytic_cases.npz")


def dev(a):
    return torch.from_numpy(np.asarray(a)).cuda().contiguous()


# Gaussian 12 of the grid case has inverse-covariance entries of 1e-4: the 1e-6 inside
# the eigenvalue square root makes its smaller eigenvalue negative, the 1e-12 floor makes
# that axis's sigma 1e6, and its integral S(x + 5e-7) - S(x - 5e-7) is then a difference
# of two fp32 numbers near 1/2 that agree to 22 bits: the reference's value and ours are
# both mostly rounding there (they differ by ~15%).  Its row is compared for finiteness only.
ILL_CONDITIONED = {"grid": [12], "flat": []}


@pytest.mark.parametrize("case", ["grid", "flat"])
def test_pixel_integral_matches_reference(cuda_device, case):
    from oss_b200 import analytic_pixel_integral

    leaves = [dev(GOLD[f"{case}_{k}"]).requires_grad_(True) for k in ("dx", "dy", "inv")]
    val = analytic_pixel_integral(*leaves)
    assert val.shape == GOLD[f"{case}_val"].shape and val.dtype == torch.float32
    keep = np.ones(GOLD[f"{case}_val"].shape[0], dtype=bool)
    keep[ILL_CONDITIONED[case]] = False
    got = val.detach().cpu().numpy()
    assert np.isfinite(got).all()
    assert_close(got[keep], GOLD[f"{case}_val"][keep], what="value")
    (val * dev(GOLD[f"{case}_up"])).sum().backward()
    for k, t in zip(("dx", "dy", "inv"), leaves):
        g = t.grad.cpu().numpy()
        assert np.isfinite(g).all()
        assert_close_grad(g[keep], GOLD[f"{case}_d_{k}"][keep], what=f"d_{k}")


def test_logistic_cdf_matches_reference(cuda_device):
    from oss_b200 import logistic_cdf

    x = dev(GOLD["cdf_x"]).requires_grad_(True)
    y = logistic_cdf(x)
    assert_close(y.detach().cpu().numpy(), GOLD["cdf_val"], what="S(x)")
    y.sum().backward()
    s = GOLD["cdf_val"].astype(np.float64)
    xs = GOLD["cdf_x"].astype(np.float64)
    assert_close(x.grad.cpu().numpy(), s * (1 - s) * (1.6 + 0.21 * xs * xs), what="S'(x)")


def test_pixel_integral_shape_errors(cuda_device):
    from oss_b200 import analytic_pixel_integral

    with pytest.raises(ValueError, match=r"sigma_2d_inv must be \(\.\.\., 2, 2\)"):
        analytic_pixel_integral(torch.zeros(3, device="cuda"), torch.zeros(3, device="cuda"),
                                torch.zeros(3, 3, device="cuda"))
