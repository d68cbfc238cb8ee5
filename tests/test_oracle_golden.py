"""Pin the CPU oracle against the reference's known answers and golden vectors.

CPU only.  Known answers come from the reference's gtests
(tests/cuda/cpp/test_preprocess.cu:67-107, test_build_pairs.cu:82-135,
test_rasterize.cu:104-164, test_rasterize_backward.cu:19-247); golden vectors
come from its PyTorch implementation (tests/golden/make_golden.py).
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import oracle as orc
from conftest import assert_close, golden_case, load_golden

RENDER = load_golden("render_cases.npz")
TIGHT = load_golden("tight_lists.npz")
OVERLAP = load_golden("overlap_cases.npz")


# --- known-answer tests from the reference gtests --------------------------------

def test_kat_preprocess_single_point_at_center():
    conic, aabb, count = orc.preprocess([[64.0, 64.0]], [[3.0, 3.0]], [0.0], 128, 128)
    assert abs(conic[0, 0] - 1.0 / 9.0) <= 1e-7 and abs(conic[0, 1]) <= 1e-7 and abs(conic[0, 2] - 1.0 / 9.0) <= 1e-7
    assert aabb[0].tolist() == [3, 3, 5, 5]
    assert count[0] == 4


def test_kat_preprocess_offscreen_and_nan_rot():
    _, aabb, count = orc.preprocess([[-100.0, -100.0], [10.0, 10.0]], [[2.0, 2.0], [3.0, 3.0]], [0.0, math.nan],
                                    128, 128)
    assert aabb.tolist() == [[0, 0, 0, 0], [0, 0, 0, 0]]
    assert count.tolist() == [0, 0]


def test_kat_build_pairs_layout():
    # test_build_pairs.cu: a 1x1 box at (2,2) of a 4-wide grid is tile 10; a 2x2
    # box at the origin covers tiles 0,1,4,5 in row-major order; no pairs -> empty.
    gid, offs = orc.pair_construction([[2, 2, 3, 3]], [1], 64, 64)
    assert gid.tolist() == [0] and offs[10] == 0 and offs[11] == 1
    gid, offs = orc.pair_construction([[0, 0, 2, 2]], [4], 64, 64)
    assert gid.tolist() == [0, 0, 0, 0]
    assert [int(offs[t + 1] - offs[t]) for t in (0, 1, 4, 5)] == [1, 1, 1, 1]
    gid, offs = orc.pair_construction([[0, 0, 0, 0]], [0], 64, 64)
    assert gid.size == 0 and int(offs[-1]) == 0


def _gauss(px, py, cx, cy, sigma):
    return math.exp(-0.5 * ((px - cx) ** 2 + (py - cy) ** 2) / sigma**2)


def test_kat_rasterize_single_and_additive():
    # test_rasterize.cu:104-164, full-frame lists; exact here instead of 5e-3.
    xy = np.array([[16.0, 16.0], [8.0, 8.0]], np.float32)
    conic = np.array([[1 / 9, 0, 1 / 9], [0.25, 0, 0.25]], np.float32)
    feat = np.array([[1.0], [2.0]], np.float32)
    gid, offs = orc.full_pairs(2, 32, 32)
    out = orc.render_forward(xy, conic, feat, gid, offs, 32, 32)
    ref = np.array([[_gauss(x, y, 16, 16, 3) + 2 * _gauss(x, y, 8, 8, 2) for x in range(32)] for y in range(32)])
    assert_close(out[0], ref, atol=1e-6, rtol=1e-6, what="additive")
    gid, offs = orc.full_pairs(1, 32, 32)
    out = orc.render_forward(xy[:1] * 0 - 100, conic[1:], feat[:1], gid, offs, 32, 32)
    assert np.abs(out).max() < 1e-30


def test_kat_backward_dfeat_and_dxy_analytic():
    # test_rasterize_backward.cu:19-207
    xy = np.array([[8.0, 8.0]], np.float32)
    conic, _, _ = orc.preprocess(xy, [[2.0, 2.0]], [0.0], 16, 16)
    gid, offs = np.array([0], np.int32), np.array([0, 1], np.int32)
    ones = np.ones((1, 16, 16), np.float32)
    _, _, d_feat, _ = orc.render_backward(xy, conic, [[1.0]], gid, offs, ones, 16, 16)
    expected = sum(_gauss(x, y, 8, 8, 2) for x in range(16) for y in range(16))
    assert abs(d_feat[0, 0] - expected) < 1e-4
    grad = np.zeros((1, 16, 16), np.float32)
    grad[0, 8, 9] = 2.0
    d_xy, d_conic, d_feat, _ = orc.render_backward(xy, [[0.25, 0.0, 0.25]], [[3.0]], gid, offs, grad, 16, 16)
    w = math.exp(-0.125)
    assert abs(d_feat[0, 0] - 2 * w) < 1e-5
    assert abs(d_xy[0, 0] - 1.5 * w) < 1e-5 and abs(d_xy[0, 1]) < 1e-5
    assert abs(d_conic[0, 0] + 3 * w) < 1e-5 and abs(d_conic[0, 1]) < 1e-5 and abs(d_conic[0, 2]) < 1e-5


def test_kat_conic_to_scale_rot():
    d_scale, d_rot = orc.conic_to_scale_rot_grad([[2.0, 4.0]], [0.0], [[3.0, 5.0, 7.0]])
    assert abs(d_scale[0, 0] + 0.75) <= 1e-6 and abs(d_scale[0, 1] + 0.21875) <= 1e-6
    assert abs(d_rot[0] - 0.9375) <= 1e-6


# --- golden vectors from the reference PyTorch implementation -------------------

@pytest.mark.parametrize("name", [str(n) for n in RENDER["names"]])
@pytest.mark.parametrize("mode", [orc.FULL, orc.EXACT])
def test_oracle_matches_reference_render(name, mode):
    c = golden_case(RENDER, name)
    h, w = (int(v) for v in c["hw"])
    img = orc.render(c["xy"], c["scale"], c["rot"], c["feat"], h, w, mode)
    assert_close(img, c["image"], what=f"image {name}")
    d_xy, d_scale, d_rot, d_feat, _, _ = orc.render_grads(c["xy"], c["scale"], c["rot"], c["feat"], c["grad"], h, w,
                                                          mode)
    assert_close(d_xy, c["d_xy"], what="d_xy")
    assert_close(d_scale, c["d_scale"], what="d_scale")
    assert_close(d_rot, c["d_rot"], what="d_rot")
    assert_close(d_feat, c["d_feat"], what="d_feat")


@pytest.mark.parametrize("name", [str(n) for n in RENDER["names"]])
def test_oracle_matches_reference_dconic(name):
    c = golden_case(RENDER, name)
    h, w = (int(v) for v in c["hw"])
    conic, _, _ = orc.preprocess(c["xy"], c["scale"], c["rot"], h, w)
    assert_close(conic, c["conic"], atol=1e-6, rtol=1e-6, what="conic")
    gid, offs = orc.full_pairs(conic.shape[0], h, w)
    _, d_conic, _, _ = orc.render_backward(c["xy"], c["conic"], c["feat"], gid, offs, c["grad"], h, w)
    assert_close(d_conic, c["d_conic"], what="d_conic")


@pytest.mark.parametrize("name", [str(n) for n in TIGHT["names"]])
def test_oracle_tight_lists_match_reference_list_builder(name):
    c = golden_case(TIGHT, name)
    h, w = (int(v) for v in c["hw"])
    conic, aabb, count, gid, offs = orc.lists(c["xy"], c["scale"], c["rot"], h, w, orc.TIGHT)
    assert_close(conic, c["conic"], atol=1e-6, rtol=1e-6, what="conic")
    np.testing.assert_array_equal(aabb, c["aabb"])
    np.testing.assert_array_equal(count, c["count"])
    np.testing.assert_array_equal(gid, c["gid"])
    np.testing.assert_array_equal(offs, c["offsets"])


def test_oracle_tile_bin_counting_sort_semantics():
    rng = np.random.default_rng(7)
    n, t = 5000, 37
    tile_id = rng.integers(-3, t + 3, size=n).astype(np.int32)
    gid = rng.integers(0, 1 << 20, size=n).astype(np.int32)
    out, offs = orc.tile_bin_counting_sort(tile_id, gid, t)
    valid = (tile_id >= 0) & (tile_id < t)
    counts = np.bincount(tile_id[valid], minlength=t)
    np.testing.assert_array_equal(offs[:t], np.concatenate([[0], np.cumsum(counts)[:-1]]))
    assert offs[t] == n
    order = np.argsort(np.where(valid, tile_id, t), kind="stable")
    np.testing.assert_array_equal(out, gid[order])


WARP = load_golden("warp_cases.npz")


def sigma_of(scales, rots):
    c, s = np.cos(rots.astype(np.float64)), np.sin(rots.astype(np.float64))
    r = np.stack([np.stack([c, -s], -1), np.stack([s, c], -1)], -2)
    d = np.zeros(r.shape)
    d[..., 0, 0] = scales[:, 0].astype(np.float64) ** 2
    d[..., 1, 1] = scales[:, 1].astype(np.float64) ** 2
    return r @ d @ np.swapaxes(r, -1, -2)


@pytest.mark.parametrize("name", [str(n) for n in WARP["names"]])
def test_oracle_warp_matches_reference(name):
    c = golden_case(WARP, name)
    pos, sc, rt, op, col, k = orc.warp_canvas(c["positions"], c["scales"], c["rotations"], c["opacities"],
                                              c["colors"], c["motion"], c["hw"], float(c["recon"]), float(c["alpha"]))
    assert k == int(c["out_count"])
    assert_close(pos, c["out_positions"], what="positions")
    assert_close(sc, c["out_scales"], atol=2e-5, what="scales")
    # rotations are compared through the covariance they parameterise (angle is
    # ill-conditioned for near-isotropic Gaussians)
    assert_close(sigma_of(sc, rt), sigma_of(c["out_scales"], c["out_rotations"]), atol=2e-5, what="covariance")
    np.testing.assert_array_equal(op, c["out_opacities"])
    np.testing.assert_array_equal(col, c["out_colors"])
    new_xy, in_frame = orc.warp_positions(c["positions"], c["pw_motion_hr"], c["hw"], float(c["alpha"]))
    assert_close(new_xy, c["pw_xy"], what="warp_positions")
    np.testing.assert_array_equal(in_frame, c["pw_in_frame"])


@pytest.mark.parametrize("name", [str(n) for n in OVERLAP["names"]])
def test_oracle_overlap_matches_reference(name):
    c = golden_case(OVERLAP, name)
    h, w = (int(v) for v in c["hw"])
    out = orc.render_overlapped_band(c["xy"], c["scale"], c["rot"], c["feat"], None, h, w, int(c["overlap"]), (0, h),
                                     grad=c["grad"], mode=orc.EXACT)
    assert_close(out["image"], c["image"], what="overlap image")
    for k in ("xy", "scale", "rot", "feat"):
        assert_close(out[f"d_{k}"][0], c[f"d_{k}"], what=f"overlap d_{k}")
        for r in out[f"d_{k}"][1]:
            assert_close(r, c[f"d_{k}"], what=f"overlap d_{k} (fp32 evaluation)")


def test_oracle_overlap_band_is_a_slice_of_the_frame():
    """A band of rows renders those rows of the whole frame, and its gradients
    are the frame's gradients under a dL/dimage that is zero off the band."""
    rng = np.random.default_rng(21)
    h, w, n, o = 70, 90, 400, 4
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    scale = np.exp(rng.standard_normal((n, 2)) * 0.5 + np.log(2.5)).astype(np.float32)
    rot = (rng.random(n) * np.pi).astype(np.float32)
    rgb = rng.random((n, 3)).astype(np.float32)
    op = rng.random(n).astype(np.float32)
    grad = rng.standard_normal((3, h, w)).astype(np.float32)
    rows = (21, 45)
    g_band = grad[:, rows[0]:rows[1]]
    full_grad = np.zeros_like(grad)
    full_grad[:, rows[0]:rows[1]] = g_band
    full = orc.render_overlapped_band(xy, scale, rot, rgb, op, h, w, o, (0, h), grad=full_grad)
    band = orc.render_overlapped_band(xy, scale, rot, rgb, op, h, w, o, rows, grad=g_band)
    np.testing.assert_array_equal(band["image"], full["image"][:, rows[0]:rows[1]])
    for k in ("d_xy", "d_scale", "d_rot", "d_feat", "d_opacity"):
        assert_close(band[k][0], full[k][0], what=k)
        assert np.abs(band[k][0]).max() > 0


@pytest.mark.parametrize("name", [str(n) for n in RENDER["names"]])
def test_oracle_fp32_evaluation_matches_reference(name):
    """The fp32 one-term-at-a-time backward (the yardstick of the gradient bar)
    against the reference's own fp32 autograd gradients, and the float64 chain
    rule against the fp32 one."""
    c = golden_case(RENDER, name)
    h, w = (int(v) for v in c["hw"])
    conic, _, _, gid, offs = orc.lists(c["xy"], c["scale"], c["rot"], h, w, orc.EXACT)
    ref = orc.grads_with_fp32_evaluation(c["xy"], c["scale"], c["rot"], conic, c["feat"], gid, offs, c["grad"], h, w)
    for k in ("xy", "scale", "rot", "feat"):
        assert_close(ref[f"d_{k}"][0], c[f"d_{k}"], what=f"double sums d_{k}")
        # the same fp32 computation as the reference's autograd in other summation
        # orders: equal up to fp32 noise, which d_scale (x 2/s^3) and d_rot amplify
        for r in ref[f"d_{k}"][1]:
            assert_close(r, c[f"d_{k}"], atol=1e-5, rtol=1e-3, what=f"fp32 evaluation d_{k}")
    for r in ref["d_xy"][1] + ref["d_feat"][1]:
        assert r.shape in (c["d_xy"].shape, c["d_feat"].shape)
    for r in ref["d_xy"][1]:
        assert_close(r, c["d_xy"], what="fp32 evaluation d_xy")
    for r in ref["d_feat"][1]:
        assert_close(r, c["d_feat"], what="fp32 evaluation d_feat")
