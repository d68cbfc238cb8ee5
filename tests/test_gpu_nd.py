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
