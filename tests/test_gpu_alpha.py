"""blend="alpha" on the GPU against the CPU oracle (oracle/oss_oracle.c
orc_render_alpha_*): depth-ordered lists bit-exact, images / transmittance /
contributor counts and all gradients within the fp32 tolerance.

The mode has no reference implementation (the reference rasterizer is additive
only), so the oracle states the compositing contract itself; it is checked
against float64 autograd in tests/test_oracle_alpha.py.  Pixels whose skip /
clamp / stop decision lies within rounding of its threshold (the oracle's
`ambiguous` mask: the GPU's exp2 differs from libm's by a few ulp) are excluded
from pixel comparisons, and gradient tests zero dL/dimage there (a pixel's
decisions reach the gradients only through its own dL/dimage).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as orc
from conftest import assert_close, assert_close_grad

pytestmark = pytest.mark.gpu


def dev(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a), dtype=dtype).cuda().contiguous()


def host(t):
    return t.detach().cpu().numpy()


def scene(n, h, w, seed, scale_lo=1.0, scale_hi=5.0, dense=False):
    rng = np.random.default_rng(seed)
    if dense:
        xy = (np.array([w, h]) * (0.2 + 0.6 * rng.random((n, 2)))).astype(np.float32)
    else:
        xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    scale = (rng.random((n, 2)) * (scale_hi - scale_lo) + scale_lo).astype(np.float32)
    rot = (rng.random(n) * 3.1).astype(np.float32)
    feat = rng.random((n, 3)).astype(np.float32)
    op = (1.0 / (1.0 + np.exp(-rng.standard_normal(n)))).astype(np.float32)
    depth = rng.random(n).astype(np.float32)
    grad = rng.standard_normal((3, h, w)).astype(np.float32)
    return xy, scale, rot, feat, op, depth, grad


def gpu_alpha(xy, scale, rot, feat, op, depth, h, w, bg=None, mode=orc.TIGHT):
    from oss_cuda import _raster

    b = _raster.bin_gaussians(dev(xy), dev(scale), dev(rot), h, w, mode, depth=None if depth is None else dev(depth))
    bgv = _raster.background_vector(bg, feat.shape[1], torch.device("cuda"))
    img, tf, nc = _raster.render_alpha_forward(b, dev(feat), None if op is None else dev(op), bgv)
    return b, bgv, img, tf, nc


@pytest.mark.parametrize("n,h,w,depth_kind", [(1, 16, 16, "rand"), (300, 64, 96, "rand"), (2000, 96, 128, "ties"),
                                              (20_000, 32, 32, "rand"), (16_384, 540, 960, "rand")])
def test_depth_ordered_lists_bit_exact(cuda_device, n, h, w, depth_kind):
    from oss_cuda import _raster

    xy, scale, rot, _, _, depth, _ = scene(n, h, w, seed=n + 3, scale_hi=40.0 if n == 20_000 else 5.0)
    if depth_kind == "ties":
        depth = np.floor(depth * 7).astype(np.float32)
        depth[::5] = -0.0
    conic, gid_ref, offs_ref = orc.alpha_lists(xy, scale, rot, depth, h, w)
    b = _raster.bin_gaussians(dev(xy), dev(scale), dev(rot), h, w, orc.TIGHT, depth=dev(depth))
    np.testing.assert_array_equal(host(b.tile_offsets), offs_ref)
    np.testing.assert_array_equal(host(b.gid_sorted), gid_ref)


def test_depth_order_permutation(cuda_device):
    from oss_cuda import _raster

    rng = np.random.default_rng(9)
    d = rng.standard_normal(70_000).astype(np.float32)
    d[::7] = 0.0
    d[3::11] = -0.0
    d[5] = np.inf
    d[6] = -np.inf
    order, rank = _raster.depth_order(dev(d))
    want = np.lexsort((np.arange(d.size), d + np.float32(0.0)))
    np.testing.assert_array_equal(host(order), want)
    np.testing.assert_array_equal(host(rank)[want], np.arange(d.size))


@pytest.mark.parametrize("n,h,w,bg,dense", [(64, 48, 64, None, False), (800, 96, 128, [0.1, 0.5, 0.9], True),
                                            (4000, 130, 170, 0.25, True), (16_384, 540, 960, None, False)])
def test_alpha_forward_matches_oracle(cuda_device, n, h, w, bg, dense):
    xy, scale, rot, feat, op, depth, _ = scene(n, h, w, seed=n, dense=dense)
    _, _, img, tf, nc = gpu_alpha(xy, scale, rot, feat, op, depth, h, w, bg)
    conic, gid, offs = orc.alpha_lists(xy, scale, rot, depth, h, w)
    ref, tf_ref, nc_ref, amb = orc.render_alpha_forward(xy, conic, feat, op, gid, offs, h, w, bg)
    ok = ~amb
    assert amb.mean() < 0.01
    assert_close(host(img)[:, ok], ref[:, ok], what="alpha image")
    assert_close(host(tf)[ok], tf_ref[ok], what="final transmittance")
    np.testing.assert_array_equal(host(nc)[ok], nc_ref[ok])
    assert (nc_ref > 0).any()


@pytest.mark.parametrize("n,h,w,seed,dense", [(40, 32, 48, 11, False), (600, 64, 80, 12, True),
                                              (3000, 96, 112, 13, True)])
def test_alpha_backward_matches_oracle(cuda_device, n, h, w, seed, dense):
    from oss_cuda import _raster

    xy, scale, rot, feat, op, depth, grad = scene(n, h, w, seed=seed, dense=dense)
    bg = [0.3, 0.1, 0.6]
    conic, gid, offs = orc.alpha_lists(xy, scale, rot, depth, h, w)
    _, _, _, amb = orc.render_alpha_forward(xy, conic, feat, op, gid, offs, h, w, bg)
    assert amb.mean() < 0.01
    grad[:, amb] = 0.0
    b, bgv, img, tf, nc = gpu_alpha(xy, scale, rot, feat, op, depth, h, w, bg)
    g = _raster.render_alpha_backward(b, dev(feat), dev(op), bgv, dev(scale), dev(rot), tf, nc, dev(grad))
    d_xy, d_conic, d_feat, d_op = orc.render_alpha_backward(xy, conic, feat, op, gid, offs, grad, h, w, bg)
    d_scale, d_rot = orc.conic_to_scale_rot_grad(scale, rot, d_conic)
    for got, want, name in ((g[0], d_xy, "d_xy"), (g[1], d_conic, "d_conic"), (g[2], d_feat, "d_feat"),
                            (g[3], d_op, "d_opacity"), (g[4], d_scale, "d_scale"), (g[5], d_rot, "d_rot")):
        assert_close_grad(host(got), want, what=name)


def test_alpha_backward_deterministic(cuda_device):
    from oss_cuda import _raster

    h, w, n = 128, 160, 5000
    xy, scale, rot, feat, op, depth, grad = scene(n, h, w, seed=21, dense=True)
    outs = []
    for _ in range(2):
        b, bgv, img, tf, nc = gpu_alpha(xy, scale, rot, feat, op, depth, h, w, 0.5)
        g = _raster.render_alpha_backward(b, dev(feat), dev(op), bgv, dev(scale), dev(rot), tf, nc, dev(grad))
        outs.append([host(img)] + [host(t) for t in g])
    for a, c in zip(*outs):
        np.testing.assert_array_equal(a, c)


def test_alpha_early_stop_known_answer(cuda_device):
    n, h, w = 30, 16, 16
    xy = np.full((n, 2), 8.0, np.float32)
    scale = np.full((n, 2), 6.0, np.float32)
    rot = np.zeros(n, np.float32)
    feat = np.tile(np.array([[1.0, 0.5, 0.25]], np.float32), (n, 1))
    op = np.full(n, 0.98, np.float32)  # T = 1 -> 0.02 -> 4e-4; a third layer would take it below 1e-4
    _, _, img, tf, nc = gpu_alpha(xy, scale, rot, feat, op, np.arange(n, dtype=np.float32), h, w)
    a = np.float64(np.float32(0.98))
    assert int(host(nc)[8, 8]) == 2
    np.testing.assert_allclose(host(tf)[8, 8], (1 - a) ** 2, rtol=1e-5)
    np.testing.assert_allclose(host(img)[:, 8, 8], feat[0] * (a + a * (1 - a)), rtol=1e-5)


def test_alpha_public_api_autograd(cuda_device):
    from oss_cuda import rasterize_gaussians

    h, w, n = 72, 88, 700
    xy, scale, rot, feat, op, depth, grad = scene(n, h, w, seed=31, dense=True)
    bg = [0.2, 0.4, 0.0]
    conic, gid, offs = orc.alpha_lists(xy, scale, rot, depth, h, w, orc.EXACT)
    _, _, _, amb = orc.render_alpha_forward(xy, conic, feat, op, gid, offs, h, w, bg)
    assert amb.mean() < 0.01
    grad[:, amb] = 0.0
    leaves = [dev(a).requires_grad_(True) for a in (xy, scale, rot, feat, op)]
    img = rasterize_gaussians(leaves[0], leaves[1], leaves[2], leaves[3], h, w, opacity=leaves[4], blend="alpha",
                              depth=dev(depth), background=bg, binning="exact")
    ref = orc.render_alpha(xy, scale, rot, feat, op, h, w, depth, bg, orc.EXACT)[0]
    assert_close(host(img)[:, ~amb], ref[:, ~amb], what="alpha image (public API)")
    gr = torch.autograd.grad(img, leaves, dev(grad))
    want = orc.render_alpha_grads(xy, scale, rot, feat, op, grad, h, w, depth, bg, orc.EXACT)
    for got, exp, name in zip(gr, (want[0], want[1], want[2], want[3], want[4]),
                              ("d_xy", "d_scale", "d_rot", "d_feat", "d_opacity")):
        assert_close_grad(host(got), exp, what=name)


def test_alpha_kwargs_validation(cuda_device):
    from oss_cuda import rasterize_gaussians

    z = torch.zeros((4, 2), device="cuda")
    r = torch.zeros((4,), device="cuda")
    f = torch.zeros((4, 3), device="cuda")
    with pytest.raises(ValueError):
        rasterize_gaussians(z, z + 1, r, f, 16, 16, depth=r)
    with pytest.raises(ValueError):
        rasterize_gaussians(z, z + 1, r, f, 16, 16, blend="over")
    with pytest.raises(RuntimeError, match="background"):
        rasterize_gaussians(z, z + 1, r, f, 16, 16, blend="alpha", background=[1.0, 2.0])
    far = z - 1000.0  # no Gaussian reaches the frame: every pixel shows the background
    out = rasterize_gaussians(far, z + 1, r, f, 16, 16, blend="alpha", background=0.5)
    np.testing.assert_allclose(host(out), 0.5, rtol=0, atol=0)
