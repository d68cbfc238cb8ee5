"""GPU canvas warp against the reference's warp_canvas golden vectors and the
CPU oracle at BASELINE config 3 size (N=200k, LR motion 540x960 -> 1080p,
alpha in {1.0, 0.5})."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle as orc
from conftest import assert_close, golden_case, load_golden

pytestmark = pytest.mark.gpu


def sigma_of(scales, rots):
    c, s = np.cos(rots.astype(np.float64)), np.sin(rots.astype(np.float64))
    r = np.stack([np.stack([c, -s], -1), np.stack([s, c], -1)], -2)
    d = np.zeros(r.shape)
    d[..., 0, 0] = scales[:, 0].astype(np.float64) ** 2
    d[..., 1, 1] = scales[:, 1].astype(np.float64) ** 2
    return r @ d @ np.swapaxes(r, -1, -2)


def canvas_of(c, device):
    from oss_b200 import CanvasState

    t = lambda k: torch.from_numpy(np.ascontiguousarray(c[k])).to(device)
    return CanvasState(t("positions"), t("scales"), t("rotations"), t("opacities"), t("colors"),
                       int(c["positions"].shape[0]))


def smooth_motion(h, w, seed, max_mag=16.0):
    """Sum of 8 random sinusoids per channel, frequencies <= 1/64 px^-1, max |m| <= max_mag."""
    rng = np.random.default_rng(seed)
    yy, xx = np.meshgrid(np.arange(h, dtype=np.float64), np.arange(w, dtype=np.float64), indexing="ij")
    out = np.zeros((2, h, w))
    for ch in range(2):
        amp = rng.random(8)
        fx = (rng.random(8) - 0.5) * (2.0 / 64.0)
        fy = (rng.random(8) - 0.5) * (2.0 / 64.0)
        ph = rng.random(8) * 2 * math.pi
        field = sum(amp[k] * np.sin(2 * math.pi * (fx[k] * xx + fy[k] * yy) + ph[k]) for k in range(8))
        out[ch] = field / amp.sum() * max_mag
    return out.astype(np.float32)


@torch.no_grad()
def test_warp_matches_reference_golden(cuda_device):
    from oss_b200 import warp_canvas, warp_positions

    data = load_golden("warp_cases.npz")
    for name in data["names"]:
        c = golden_case(data, str(name))
        hw = tuple(int(v) for v in c["hw"])
        motion = torch.from_numpy(c["motion"]).to(cuda_device)
        out = warp_canvas(canvas_of(c, cuda_device), motion, hw, sigma_recon=float(c["recon"]),
                          alpha=float(c["alpha"]))
        assert out.count == int(c["out_count"])
        assert_close(out.positions.cpu().numpy(), c["out_positions"], what=f"{name} positions")
        assert_close(out.scales.cpu().numpy(), c["out_scales"], atol=2e-5, what=f"{name} scales")
        assert_close(sigma_of(out.scales.cpu().numpy(), out.rotations.cpu().numpy()),
                     sigma_of(c["out_scales"], c["out_rotations"]), atol=2e-5, what=f"{name} covariance")
        np.testing.assert_array_equal(out.opacities.cpu().numpy(), c["out_opacities"])
        np.testing.assert_array_equal(out.colors.cpu().numpy(), c["out_colors"])
        new_xy, in_frame = warp_positions(torch.from_numpy(c["positions"]).to(cuda_device),
                                          torch.from_numpy(c["pw_motion_hr"]).to(cuda_device), hw,
                                          alpha=float(c["alpha"]))
        assert_close(new_xy.cpu().numpy(), c["pw_xy"], what=f"{name} warp_positions")
        np.testing.assert_array_equal(in_frame.cpu().numpy(), c["pw_in_frame"])


@pytest.mark.parametrize("alpha", [1.0, 0.5])
@torch.no_grad()
def test_warp_config3_size_matches_oracle(cuda_device, alpha):
    from oss_b200 import CanvasState, warp_canvas

    n, h, w, hl, wl = 200_000, 1080, 1920, 540, 960
    rng = np.random.default_rng(33)
    pos = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    sc = np.exp(rng.standard_normal((n, 2)) * 0.3 + math.log(2.0)).astype(np.float32)
    rt = (rng.random(n) * math.pi).astype(np.float32)
    op = (1 / (1 + np.exp(-rng.standard_normal(n)))).astype(np.float32)
    col = rng.random((n, 3)).astype(np.float32)
    motion = smooth_motion(hl, wl, seed=34)
    r_pos, r_sc, r_rt, r_op, r_col, r_k = orc.warp_canvas(pos, sc, rt, op, col, motion[None], (h, w), 0.5, alpha)
    t = lambda a: torch.from_numpy(a).to(cuda_device)
    out = warp_canvas(CanvasState(t(pos), t(sc), t(rt), t(op), t(col), n), t(motion[None]), (h, w), 0.5, alpha)
    assert out.count == r_k and 0 < r_k < n
    # same op order on both sides: positions, compaction order and carried fields are bit-exact
    np.testing.assert_array_equal(out.positions.cpu().numpy(), r_pos)
    np.testing.assert_array_equal(out.opacities.cpu().numpy(), r_op)
    np.testing.assert_array_equal(out.colors.cpu().numpy(), r_col)
    assert_close(out.scales.cpu().numpy(), r_sc, atol=2e-5, what="scales")
    assert_close(sigma_of(out.scales.cpu().numpy(), out.rotations.cpu().numpy()), sigma_of(r_sc, r_rt), atol=2e-5,
                 what="covariance")


@torch.no_grad()
def test_warp_identity_and_empty(cuda_device):
    from oss_b200 import CanvasState, warp_canvas

    n = 1000
    rng = np.random.default_rng(5)
    pos = torch.from_numpy((rng.random((n, 2)) * 64).astype(np.float32)).to(cuda_device)
    sc = torch.from_numpy((rng.random((n, 2)) + 0.5).astype(np.float32)).to(cuda_device)
    rt = torch.from_numpy((rng.random(n) * 3).astype(np.float32)).to(cuda_device)
    op = torch.rand(n, device=cuda_device)
    col = torch.rand(n, 8, device=cuda_device)
    canvas = CanvasState(pos, sc, rt, op, col, n)
    out = warp_canvas(canvas, torch.zeros(1, 2, 32, 32, device=cuda_device), (64, 64))
    assert out.count == n
    assert torch.equal(out.positions, pos) and torch.equal(out.scales, sc) and torch.equal(out.rotations, rt)
    empty = warp_canvas(CanvasState(pos, sc, rt, op, col, 0), torch.zeros(1, 2, 8, 8, device=cuda_device), (64, 64))
    assert empty.count == 0 and empty.positions.shape == (0, 2)


def test_warp_refuses_grad_inputs(cuda_device):
    from oss_b200 import CanvasState, warp_canvas

    pos = torch.rand(4, 2, device=cuda_device, requires_grad=True)
    canvas = CanvasState(pos, torch.ones(4, 2, device=cuda_device), torch.zeros(4, device=cuda_device),
                         torch.ones(4, device=cuda_device), torch.ones(4, 3, device=cuda_device), 4)
    with pytest.raises(RuntimeError, match="forward-only"):
        warp_canvas(canvas, torch.zeros(1, 2, 8, 8, device=cuda_device), (16, 16))
