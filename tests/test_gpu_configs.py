"""Parity at the full sizes of the BASELINE configs that the bench times beyond
config 2: config 4 (2160x3840, N=1M, feathered overlap 4 with a spawner offset,
fwd+bwd), config 5 (one 1080p frame of an own 200k canvas plus a shared 50k
canvas, and the shared canvas's gradients summed over frames), and the
blend="alpha" mode at config-2 size.

Gradients are held to the parity bar against the oracle's float64 sums; an
element outside it passes only beside float64 evidence that the reference's
own fp32 evaluation is that far off as well (conftest.assert_close_grad).
"""
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


def host(t):
    return t.detach().cpu().numpy()


def gaussians(n, h, w, seed, log_scale_mean, log_scale_sd):
    """BASELINE distributions: means uniform over the frame, log-scales normal
    per axis, rotation U[0, pi), opacity sigmoid(N(0, 1)), rgb U[0, 1]."""
    rng = np.random.default_rng(seed)
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    scale = np.exp(rng.standard_normal((n, 2)) * log_scale_sd + log_scale_mean).astype(np.float32)
    rot = (rng.random(n) * math.pi).astype(np.float32)
    op = (1.0 / (1.0 + np.exp(-rng.standard_normal(n)))).astype(np.float32)
    rgb = rng.random((n, 3)).astype(np.float32)
    return xy, scale, rot, op, rgb


def check_grads(got: dict, ref: dict, prefix: str):
    for name, value in got.items():
        truth, fp32 = ref[name]
        assert_close_grad(value, truth, what=f"{prefix}{name}", ref32=fp32)


def autograd(xy, scale, rot, rgb, op, grad, h, w, **kw):
    from oss_cuda import rasterize_gaussians

    leaves = [dev(a).requires_grad_(True) for a in (xy, scale, rot, rgb, op)]
    img = rasterize_gaussians(leaves[0], leaves[1], leaves[2], leaves[3], h, w, opacity=leaves[4], **kw)
    img.backward(dev(grad))
    names = ("d_xy", "d_scale", "d_rot", "d_feat", "d_opacity")
    return host(img), {k: host(t.grad) for k, t in zip(names, leaves)}


def test_config4_feathered_overlap_band(cuda_device):
    """Config 4 at full size: a 2160x3840 frame of 1M Gaussians (log-scale
    ln 2.5, sd 0.5), overlap 4, spawner offset (7, 11), 3-sigma lists, fwd+bwd.
    The oracle composes its four phase renders with the reference's feather
    formula over a band of 40 rows that crosses tile edges of every phase;
    dL/dimage is zero off the band, so every gradient is the band's."""
    h, w, n, overlap, offset = 2160, 3840, 1_000_000, 4, (7, 11)
    xy, scale, rot, op, rgb = gaussians(n, h, w, 44, math.log(2.5), 0.5)
    rows = (1000, 1040)
    g_band = np.random.default_rng(45).standard_normal((3, rows[1] - rows[0], w)).astype(np.float32)
    grad = np.zeros((3, h, w), np.float32)
    grad[:, rows[0]:rows[1]] = g_band
    img, got = autograd(xy, scale, rot, rgb, op, grad, h, w, binning="tight3sigma", overlap=overlap,
                        phase_offset=offset)
    xy_off = (xy + np.array(offset, np.float32)).astype(np.float32)  # the API's fp32 offset add
    ref = orc.render_overlapped_band(xy_off, scale, rot, rgb, op, h, w, overlap, rows, grad=g_band)
    assert_close(img[:, rows[0]:rows[1]], ref["image"], what="config4 band image")
    assert float(np.abs(ref["image"]).max()) > 0.1
    check_grads(got, ref, "config4 ")
    touched = np.abs(ref["d_feat"][0]).sum(1) > 0
    assert touched.sum() > 10_000  # the band reaches many Gaussians
    assert np.all(got["d_feat"][~touched] == 0.0)


def test_config5_own_and_shared_canvas(cuda_device):
    """Config 5: frames of an own 200k canvas plus a shared 50k canvas rendered
    together (250k Gaussians, 1080p, fwd+bwd).  Frame 0's image and gradients
    against the oracle, then the shared canvas's gradients summed over two
    frames (as the all-reduce of the batched step sums them) against the sum
    of the oracle's."""
    from oss_b200.distributed import SHARED_GRAD_FIELDS

    h, w, n_own, n_sh = 1080, 1920, 200_000, 50_000
    shared = gaussians(n_sh, h, w, 555, math.log(2.0), 0.3)
    sl = slice(n_own, n_own + n_sh)
    names = [name for name, _ in SHARED_GRAD_FIELDS]
    sum_got = {k: 0.0 for k in names}
    sum_truth = {k: 0.0 for k in names}
    sum_fp32 = {k: [0.0, 0.0] for k in names}
    for frame in range(2):
        own = gaussians(n_own, h, w, 10_000 + frame, math.log(2.0), 0.3)
        xy, scale, rot, op, rgb = (np.concatenate([a, b]) for a, b in zip(own, shared))
        grad = np.random.default_rng(70 + frame).standard_normal((3, h, w)).astype(np.float32)
        img, got = autograd(xy, scale, rot, rgb, op, grad, h, w, binning="tight3sigma")
        got["d_rgb"] = got.pop("d_feat")
        conic, _, _, gid, offs = orc.lists(xy, scale, rot, h, w, orc.TIGHT)
        ref = orc.grads_with_fp32_evaluation(xy, scale, rot, conic, rgb, gid, offs, grad, h, w, op)
        ref["d_rgb"] = ref.pop("d_feat")
        if frame == 0:
            assert_close(img, orc.render_forward(xy, conic, rgb, gid, offs, h, w, op), what="config5 image")
            check_grads(got, ref, "config5 frame 0 ")
        for k in names:
            sum_got[k] = sum_got[k] + got[k][sl].astype(np.float64)
            sum_truth[k] = sum_truth[k] + ref[k][0][sl].astype(np.float64)
            sum_fp32[k] = [acc + r[sl].astype(np.float64) for acc, r in zip(sum_fp32[k], ref[k][1])]
    for k in names:
        assert_close_grad(sum_got[k], sum_truth[k], what=f"config5 shared {k} over 2 frames", ref32=sum_fp32[k])


def test_alpha_blend_config2_size(cuda_device):
    """blend="alpha" at config-2 size (1080p, 200k, depth U[0, 1]): depth-ordered
    lists bit-exact, image / transmittance / contributor counts, and every
    gradient against the oracle (pixels whose skip / clamp / stop test lies
    within rounding of its threshold are left out, and their dL/dimage is 0)."""
    from oss_cuda import _raster

    h, w, n = 1080, 1920, 200_000
    xy, scale, rot, op, rgb = gaussians(n, h, w, 909, math.log(2.0), 0.3)
    rng = np.random.default_rng(910)
    depth = rng.random(n).astype(np.float32)
    grad = rng.standard_normal((3, h, w)).astype(np.float32)
    conic, gid, offs = orc.alpha_lists(xy, scale, rot, depth, h, w)
    ref, tf_ref, nc_ref, amb = orc.render_alpha_forward(xy, conic, rgb, op, gid, offs, h, w)
    assert amb.mean() < 0.01
    b = _raster.bin_gaussians(dev(xy), dev(scale), dev(rot), h, w, orc.TIGHT, depth=dev(depth))
    np.testing.assert_array_equal(host(b.tile_offsets), offs)
    np.testing.assert_array_equal(host(b.gid_sorted), gid)
    bgv = _raster.background_vector(None, 3, torch.device("cuda"))
    img, tf, nc = _raster.render_alpha_forward(b, dev(rgb), dev(op), bgv)
    ok = ~amb
    assert_close(host(img)[:, ok], ref[:, ok], what="alpha config2 image")
    assert_close(host(tf)[ok], tf_ref[ok], what="alpha config2 transmittance")
    np.testing.assert_array_equal(host(nc)[ok], nc_ref[ok])
    grad[:, amb] = 0.0
    g = _raster.render_alpha_backward(b, dev(rgb), dev(op), bgv, dev(scale), dev(rot), tf, nc, dev(grad))
    d_xy, d_conic, d_feat, d_op = orc.render_alpha_backward(xy, conic, rgb, op, gid, offs, grad, h, w)
    d_scale, d_rot = orc.conic_to_scale_rot_grad_f64(scale, rot, d_conic)
    for got, want, name in ((g[0], d_xy, "d_xy"), (g[1], d_conic, "d_conic"), (g[2], d_feat, "d_feat"),
                            (g[3], d_op, "d_opacity"), (g[4], d_scale, "d_scale"), (g[5], d_rot, "d_rot")):
        assert_close_grad(host(got), want, what=f"alpha config2 {name}")
