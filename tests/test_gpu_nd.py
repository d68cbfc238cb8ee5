"""v7 N-D time-slice rasterizer on the GPU (oss_b200.render_nd_time_slice over
csrc/nd.cu) against the reference's own forward and autograd
(tests/golden/nd_cases.npz, made by tests/golden/make_nd_golden.py): image within
1e-5 abs / 1e-4 rel, gradients of means, covariances, features and opacities
within the same bar plus 1e-6 of each tensor's largest magnitude (fp32 sums)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import assert_close, assert_close_grad

pytestmark = pytest.mark.gpu

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "nd_cases.npz")


def dev(a):
    return torch.from_numpy(np.asarray(a)).cuda().contiguous()


@pytest.mark.parametrize("name", ["a", "b", "c", "d"])
def test_nd_time_slice_matches_reference(cuda_device, name):
    from oss_b200 import render_nd_time_slice

    h, w, tq, falloff, v3, v2 = GOLD[name + "_args"]
    leaves = [dev(GOLD[f"{name}_{k}"]).requires_grad_(True) for k in ("means", "covs", "feats", "opac")]
    img = render_nd_time_slice(leaves[0], leaves[1], leaves[2], leaves[3], float(tq), (int(h), int(w)),
                               time_falloff=bool(falloff), mip_3d_variance=float(v3), mip_2d_variance=float(v2))
    assert img.shape == GOLD[name + "_img"].shape
    assert_close(img.detach().cpu().numpy(), GOLD[name + "_img"], what="image")
    (img * dev(GOLD[name + "_up"])).sum().backward()
    for k, t in zip(("means", "covs", "feats", "opac"), leaves):
        assert_close_grad(t.grad.cpu().numpy(), GOLD[f"{name}_d_{k}"], what=f"d_{k}")


def test_nd_empty_and_offscreen(cuda_device):
    from oss_b200 import render_nd_time_slice

    covs = torch.eye(3, device="cuda").repeat(3, 1, 1)
    means = torch.tensor([[-50.0, -50.0, 0.5], [500.0, 10.0, 0.5], [10.0, 10.0, 0.5]], device="cuda")
    feats = torch.ones((3, 2), device="cuda")
    op = torch.full((3,), 0.5, device="cuda")
    img = render_nd_time_slice(means[:2], covs[:2], feats[:2], op[:2], 0.5, (32, 32))
    assert img.shape == (2, 32, 32) and not img.any()
    img = render_nd_time_slice(means, covs, feats, op, 0.5, (32, 32))
    assert float(img.max()) > 0.0
    z = render_nd_time_slice(means[:0], covs[:0], feats[:0], op[:0], 0.5, (16, 16))
    assert z.shape == (2, 16, 16) and not z.any()


def _condition_f64(means, covs, opac, tq, falloff, v3, v2):
    """The conditioning steps in float64 PyTorch ops (test oracle for the fused kernel's
    forward and hand-written backward): Mip 3D smoothing, Schur complement at t_query,
    Mip 2D filter, inverse covariance (a, b, d) and amplitude."""
    eye3 = torch.eye(3, dtype=torch.float64, device=means.device)
    S, opf = covs, opac
    if v3 > 0:
        S = covs + v3 * eye3
        opf = opac * torch.sqrt(torch.det(covs).clamp(min=1e-12) / torch.det(S).clamp(min=1e-12))
    vtt = S[:, 2, 2].clamp(min=1e-12)
    vxt = S[:, :2, 2]
    dt = tq - means[:, 2]
    xy = means[:, :2] + vxt * (dt / vtt)[:, None]
    c = S[:, :2, :2] - vxt[:, :, None] * vxt[:, None, :] / vtt[:, None, None]
    wt = torch.exp(-0.5 * dt * dt / vtt - 0.5 * (np.log(2 * np.pi) + torch.log(vtt)))
    W = wt if falloff else torch.ones_like(wt)
    P = c
    if v2 > 0:
        P = c + v2 * torch.eye(2, dtype=torch.float64, device=means.device)
        W = W * torch.sqrt(torch.det(c).clamp(min=1e-12) / torch.det(P).clamp(min=1e-12))
    inv = torch.linalg.inv(P)
    return xy, torch.stack([inv[:, 0, 0], inv[:, 0, 1], inv[:, 1, 1]], -1), opf * W


@pytest.mark.parametrize("falloff,v3,v2", [(True, 0.2, 0.1), (False, 0.0, 0.0), (True, 0.0, 0.3), (True, 0.5, 0.0)])
def test_nd_condition_kernel_and_chain_rule(cuda_device, falloff, v3, v2):
    """The fused conditioning kernel and its hand-written backward against float64
    autograd, on 5,000 random Gaussians (non-symmetric covariance inputs included:
    each of the nine entries gets its own gradient, as in the reference)."""
    from oss_b200.nd import _NDCondition

    g = torch.Generator(device="cpu").manual_seed(13)
    n = 5000
    L = torch.tril(torch.randn(n, 3, 3, generator=g, dtype=torch.float64)) * torch.tensor([1.5, 1.2, 0.3],
                                                                                          dtype=torch.float64)[:, None]
    covs = L @ L.transpose(1, 2) + torch.diag(torch.tensor([0.4, 0.4, 0.03], dtype=torch.float64))
    covs = covs + 0.01 * torch.randn(n, 3, 3, generator=g, dtype=torch.float64)  # slightly non-symmetric
    means = torch.rand(n, 3, generator=g, dtype=torch.float64) * torch.tensor([60.0, 40.0, 1.0], dtype=torch.float64)
    opac = torch.rand(n, generator=g, dtype=torch.float64) * 0.9 + 0.05
    gxy, gcon, gamp = (torch.randn(n, 2, generator=g, dtype=torch.float64), torch.randn(n, 3, generator=g,
                       dtype=torch.float64), torch.randn(n, generator=g, dtype=torch.float64))
    leaves64 = [t.cuda().requires_grad_(True) for t in (means, covs, opac)]
    r64 = _condition_f64(*leaves64, 0.4, falloff, v3, v2)
    sum(((a * b.cuda()).sum() for a, b in zip(r64, (gxy, gcon, gamp)))).backward()
    leaves32 = [t.float().cuda().requires_grad_(True) for t in (means, covs, opac)]
    xy, conic, amp, box = _NDCondition.apply(*leaves32, 0.4, falloff, v3, v2, 40, 60)
    for got, ref, what in zip((xy, conic, amp), r64, ("xy", "conic", "amp")):
        assert_close(got.detach().cpu().numpy(), ref.detach().cpu().numpy(), atol=1e-5, rtol=2e-4, what=what)
    sum(((a * b.float().cuda()).sum() for a, b in zip((xy, conic, amp), (gxy, gcon, gamp)))).backward()
    for t32, t64, what in zip(leaves32, leaves64, ("d_means", "d_covs", "d_opac")):
        ref = t64.grad.cpu().numpy()
        assert_close(t32.grad.cpu().numpy(), ref, atol=1e-4 + 1e-5 * float(np.abs(ref).max()), rtol=1e-3, what=what)
