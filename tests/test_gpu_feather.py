"""The one-pass feathered overlapping-tile render (rasterize_gaussians(overlap=o),
csrc/feather.cu) against the oracle's composition of the reference's four
phase renders (oss/sr/v6/rasterizer.py:159-242, oracle.render_overlapped_band):
images and all gradients, over overlaps, channel counts, list modes and frame
sizes that cut tiles, with Gaussians placed where the reference's shifted
means x + o round in fp32 (just below powers of two, and within o of 0)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle as orc
from conftest import assert_close, assert_close_grad

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32).cuda()


def scene(n, h, w, f, seed, overlap):
    rng = np.random.default_rng(seed)
    xy = (rng.random((n, 2)) * np.array([w + 20, h + 20]) - 10).astype(np.float32)
    # a quarter of the means just below powers of two, an eighth within `overlap` of 0:
    # there fl(x + o) rounds and the shifted phases evaluate a second centre
    k = n // 4
    pw = np.array([p for p in (8, 16, 32, 64, 128, 256) if p < max(h, w)], np.float32)
    xy[:k] = pw[rng.integers(0, pw.size, (k, 2))] - (rng.random((k, 2)) * overlap).astype(np.float32)
    xy[k:k + k // 2] = (rng.random((k // 2, 2)) * overlap).astype(np.float32)
    scale = np.exp(rng.standard_normal((n, 2)) * 0.5 + math.log(2.0)).astype(np.float32)
    rot = (rng.random(n) * math.pi).astype(np.float32)
    feat = (rng.random((n, f)) - 0.3).astype(np.float32)
    op = rng.random(n).astype(np.float32)
    grad = rng.standard_normal((f, h, w)).astype(np.float32)
    return xy, scale, rot, feat, op, grad


def shifted_inexact(xy, overlap):
    x1 = (xy + np.float32(overlap)).astype(np.float32)
    back = (x1 - np.float32(overlap)).astype(np.float32)
    return int(np.any(back != xy, axis=1).sum())


def run(xy, scale, rot, feat, op, grad, h, w, overlap, binning):
    from oss_cuda import rasterize_gaussians

    leaves = [dev(a).requires_grad_(True) for a in (xy, scale, rot, feat, op)]
    img = rasterize_gaussians(leaves[0], leaves[1], leaves[2], leaves[3], h, w, binning=binning,
                              opacity=leaves[4], overlap=overlap)
    img.backward(dev(grad))
    names = ("d_xy", "d_scale", "d_rot", "d_feat", "d_opacity")
    return img.detach().cpu().numpy(), {k: t.grad.cpu().numpy() for k, t in zip(names, leaves)}


CASES = [  # n, h, w, f, overlap, binning
    (600, 70, 150, 3, 4, "tight3sigma"),
    (900, 130, 97, 1, 4, "exact"),
    (500, 64, 64, 5, 1, "tight3sigma"),
    (700, 81, 140, 12, 7, "tight3sigma"),
    (400, 100, 90, 16, 15, "exact"),
    (500, 90, 120, 3, 16, "tight3sigma"),
    (500, 90, 120, 4, 20, "tight3sigma"),
    (300, 33, 47, 8, 4, "full"),
]


@pytest.mark.parametrize("n,h,w,f,overlap,binning", CASES)
def test_feathered_one_pass_matches_phase_composition(cuda_device, n, h, w, f, overlap, binning):
    from oss_cuda import _feather

    assert _feather.supported(overlap, f, h, w)
    xy, scale, rot, feat, op, grad = scene(n, h, w, f, seed=n + 31 * overlap + f, overlap=overlap)
    assert shifted_inexact(xy, overlap) > 10  # the variant path is exercised
    img, got = run(xy, scale, rot, feat, op, grad, h, w, overlap, binning)
    ref = orc.render_overlapped_band(xy, scale, rot, feat, op, h, w, overlap, (0, h), grad=grad,
                                     mode=orc.MODES[binning])
    assert_close(img, ref["image"], what="image")
    assert float(np.abs(ref["image"]).max()) > 0.05
    for k, v in got.items():
        truth, fp32 = ref[k]
        assert_close_grad(v, truth, what=k, ref32=fp32)


def test_feathered_one_pass_agrees_with_composition_path(cuda_device):
    """The one-pass render and the four-render composition of the same kernels
    (what the call falls back to beyond 16 channels) give the same image."""
    from oss_cuda import rasterize_gaussians
    from oss_cuda.overlap import render_overlapped_with

    h, w, n, o = 200, 260, 5000, 4
    xy, scale, rot, feat, op, _ = scene(n, h, w, 3, seed=3, overlap=o)
    t = [dev(a) for a in (xy, scale, rot, feat, op)]
    one = rasterize_gaussians(t[0], t[1], t[2], t[3], h, w, binning="tight3sigma", opacity=t[4], overlap=o)

    def render(x, s, r, f, hh, ww):
        return rasterize_gaussians(x, s, r, f, hh, ww, binning="tight3sigma", opacity=t[4])

    four = render_overlapped_with(render, t[0], t[1], t[2], t[3], h, w, o)
    assert_close(one.cpu().numpy(), four.cpu().numpy(), what="one pass vs four renders")


def test_feathered_wide_channels_fall_back(cuda_device):
    """Above 16 channels the call composes four renders (still on the GPU kernels)."""
    from oss_cuda import _feather, rasterize_gaussians

    h, w, n, o, f = 48, 64, 300, 4, 20
    assert not _feather.supported(o, f, h, w)
    xy, scale, rot, feat, op, grad = scene(n, h, w, f, seed=9, overlap=o)
    img = rasterize_gaussians(dev(xy), dev(scale), dev(rot), dev(feat), h, w, binning="tight3sigma",
                              opacity=dev(op), overlap=o)
    ref = orc.render_overlapped_band(xy, scale, rot, feat, op, h, w, o, (0, h))
    assert_close(img.cpu().numpy(), ref["image"], what="image")


def test_feathered_sync_free_capacity(cuda_device):
    """pair_capacity: no host read; an undersized capacity empties the lists and
    raises the sticky flag instead of writing past them."""
    from oss_cuda import pair_capacity_overflowed, rasterize_gaussians

    h, w, n, o = 64, 80, 400, 4
    xy, scale, rot, feat, op, _ = scene(n, h, w, 3, seed=5, overlap=o)
    t = [dev(a) for a in (xy, scale, rot, feat, op)]
    pair_capacity_overflowed(cuda_device)
    exact = rasterize_gaussians(t[0], t[1], t[2], t[3], h, w, binning="tight3sigma", opacity=t[4], overlap=o)
    roomy = rasterize_gaussians(t[0], t[1], t[2], t[3], h, w, binning="tight3sigma", opacity=t[4], overlap=o,
                                pair_capacity=200_000)
    assert not pair_capacity_overflowed(cuda_device)
    assert torch.equal(exact, roomy)
    tiny = rasterize_gaussians(t[0], t[1], t[2], t[3], h, w, binning="tight3sigma", opacity=t[4], overlap=o,
                               pair_capacity=10)
    assert pair_capacity_overflowed(cuda_device)
    assert float(tiny.abs().max()) == 0.0
