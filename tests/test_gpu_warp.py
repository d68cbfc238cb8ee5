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


# ------------------------------------------------------------------ gradients

def warp_f64(pos, scales, rots, ops, cols, motion_lr, hw, recon):
    """The reference's canvas warp (oss/sr/v6/canvas_warp.py:177-254 with
    covariance_resampling.py:76-116) restated with the same torch operations in
    float64 on the CPU, so that autograd gives the exact-arithmetic gradients
    the GPU backward is judged against."""
    import torch.nn.functional as F

    h, w = hw
    m = motion_lr[:1]
    if tuple(m.shape[-2:]) != (h, w):
        m = F.interpolate(m, size=(h, w), mode="bilinear", align_corners=False)
    grid = torch.stack([pos[:, 0] / w * 2.0 - 1.0, pos[:, 1] / h * 2.0 - 1.0], -1).view(1, -1, 1, 2)
    sm = F.grid_sample(m, grid, mode="bilinear", padding_mode="zeros", align_corners=False)
    new_pos = pos + sm.view(2, -1).t()
    keep = (new_pos[:, 0] >= 0) & (new_pos[:, 0] < w) & (new_pos[:, 1] >= 0) & (new_pos[:, 1] < h)
    pad = F.pad(m, (1, 1, 1, 1), mode="replicate")
    dmdx = (pad[..., 1:-1, 2:] - pad[..., 1:-1, :-2]) * 0.5
    dmdy = (pad[..., 2:, 1:-1] - pad[..., :-2, 1:-1]) * 0.5
    sx = F.grid_sample(dmdx, grid, mode="bilinear", padding_mode="border", align_corners=False)[0, :, :, 0].t()
    sy = F.grid_sample(dmdy, grid, mode="bilinear", padding_mode="border", align_corners=False)[0, :, :, 0].t()
    j = torch.eye(2, dtype=pos.dtype).expand(pos.shape[0], -1, -1).clone()
    j[:, 0, 0] += sx[:, 0]
    j[:, 1, 0] += sx[:, 1]
    j[:, 0, 1] += sy[:, 0]
    j[:, 1, 1] += sy[:, 1]
    ident = (j - torch.eye(2, dtype=pos.dtype)).abs().reshape(-1, 4).amax(-1) < 1e-5
    c, s = torch.cos(rots), torch.sin(rots)
    r = torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2)
    sig = r @ torch.diag_embed(scales.clamp(min=0.0).square()) @ r.transpose(-1, -2)
    u = j @ sig @ j.transpose(-1, -2) + torch.eye(2, dtype=pos.dtype) * recon
    u = 0.5 * (u + u.transpose(-1, -2)) + 1e-7 * torch.eye(2, dtype=pos.dtype)
    u = 0.5 * (u + u.transpose(-1, -2))
    a, b, cc = u[:, 0, 0], u[:, 0, 1], u[:, 1, 1]
    ht, hd = 0.5 * (a + cc), 0.5 * (a - cc)
    rad = torch.sqrt(hd.square() + b.square() + 1e-12)
    new_sc = torch.sqrt(torch.stack([(ht + rad).clamp(min=1e-12), (ht - rad).clamp(min=1e-12)], -1))
    new_rot = 0.5 * torch.atan2(2.0 * b, a - cc)
    new_sc = torch.where(ident[:, None], scales, new_sc)
    new_rot = torch.where(ident, rots, new_rot)
    return new_pos[keep], new_sc[keep], new_rot[keep], ops[keep], cols[keep]


def _gpu_warp_grads(c, device, alpha=1.0):
    from oss_b200 import CanvasState, warp_canvas

    names = ("positions", "scales", "rotations", "opacities", "colors", "motion")
    leaves = [torch.from_numpy(np.ascontiguousarray(c[k])).to(device).requires_grad_(True) for k in names]
    hw = tuple(int(v) for v in c["hw"])
    canvas = CanvasState(*leaves[:5], count=int(leaves[0].shape[0]))
    out = warp_canvas(canvas, leaves[5], hw, sigma_recon=float(c["recon"]), alpha=alpha)
    assert out.count == int(c["out_count"])
    outs = (out.positions, out.scales, out.rotations, out.opacities, out.colors)
    loss = sum((o * torch.from_numpy(c[f"g_{k}"]).to(device)).sum() for o, k in zip(outs, names[:5]))
    loss.backward()
    return {k: t.grad.cpu().numpy() for k, t in zip(names, leaves)}


def _f64_warp_grads(c, alpha=1.0, dtype=torch.float64):
    """Autograd gradients of warp_f64 (float64: the exact value; float32: the
    reference's own fp32 arithmetic, whose floor and comparison decisions match
    the kernels' where a sample point sits within rounding of a texel edge)."""
    names = ("positions", "scales", "rotations", "opacities", "colors", "motion")
    leaves = [torch.from_numpy(np.ascontiguousarray(c[k])).to(dtype).requires_grad_(True) for k in names]
    hw = tuple(int(v) for v in c["hw"])
    outs = warp_f64(*leaves[:5], leaves[5] * alpha, hw, float(c["recon"]))
    loss = sum((o * torch.from_numpy(c[f"g_{k}"]).to(dtype)).sum() for o, k in zip(outs, names[:5]))
    loss.backward()
    return {k: t.grad.numpy() for k, t in zip(names, leaves)}


def test_warp_backward_matches_reference_autograd(cuda_device):
    """Every input's gradient (positions, scales, rotations, opacities, colors,
    motion) against the float64 restatement's autograd, with the reference's own
    fp32 autograd gradients (golden) as the fp32 yardstick; the golden values
    themselves agree with the float64 ones."""
    from conftest import assert_close_grad

    data = load_golden("warp_grad_cases.npz")
    for name in data["names"]:
        c = golden_case(data, str(name))
        got = _gpu_warp_grads(c, cuda_device)
        exact = _f64_warp_grads(c)
        for k, v in got.items():
            assert_close_grad(v, exact[k], what=f"{name} d_{k}", ref32=[c[f"d_{k}"]])
            assert_close_grad(c[f"d_{k}"], exact[k], what=f"{name} golden d_{k}", ref32=[c[f"d_{k}"]])
        assert np.abs(got["motion"]).sum() > 0


def test_warp_gradient_flow_from_positions_to_motion(cuda_device):
    """tests/sr/v6/test_canvas_warp.py:94-101 on the GPU: positions.sum()
    backward reaches motion_lr with finite, non-zero gradients -- the same
    gradients the reference computes (golden case "flow")."""
    from oss_b200 import CanvasState, warp_canvas

    c = golden_case(load_golden("warp_grad_cases.npz"), "flow")
    canvas = CanvasState(*(torch.from_numpy(np.ascontiguousarray(c[k])).to(cuda_device)
                           for k in ("positions", "scales", "rotations", "opacities", "colors")), count=3)
    motion = torch.zeros(1, 2, 32, 32, device=cuda_device, requires_grad=True)
    out = warp_canvas(canvas, motion, output_hw=(64, 64))
    out.positions.sum().backward()
    assert motion.grad is not None
    assert torch.isfinite(motion.grad).all()
    assert float(motion.grad.abs().sum()) > 0.0
    assert_close(motion.grad.cpu().numpy(), c["d_motion"], what="d_motion")


def test_warp_backward_alpha_and_size(cuda_device):
    """alpha-scaled motion and a 2x upsampling at a larger size (20k Gaussians,
    LR 135x240 -> 270x480) against the float64 restatement, and the motion
    gradient's linearity in alpha."""
    from conftest import assert_close_grad

    rng = np.random.default_rng(31)
    n, lr, hr = 20_000, (135, 240), (270, 480)
    c = {"positions": (rng.random((n, 2)) * np.array([hr[1] + 8, hr[0] + 8]) - 4).astype(np.float32),
         "scales": np.exp(rng.standard_normal((n, 2)) * 0.4 + math.log(1.5)).astype(np.float32),
         "rotations": (rng.random(n) * math.pi).astype(np.float32),
         "opacities": rng.random(n).astype(np.float32), "colors": rng.random((n, 3)).astype(np.float32),
         "motion": smooth_motion(lr[0], lr[1], 77, max_mag=6.0)[None], "hw": np.array(hr), "recon": 0.5}
    alpha = 0.5
    with torch.no_grad():
        from oss_b200 import CanvasState, warp_canvas

        k = warp_canvas(CanvasState(*(torch.from_numpy(c[key]).to(cuda_device) for key in
                                      ("positions", "scales", "rotations", "opacities", "colors")), count=n),
                        torch.from_numpy(c["motion"]).to(cuda_device), hr, 0.5, alpha=alpha).count
    c["out_count"] = k
    for key, shape in (("positions", (k, 2)), ("scales", (k, 2)), ("rotations", (k,)), ("opacities", (k,)),
                       ("colors", (k, 3))):
        c[f"g_{key}"] = rng.standard_normal(shape).astype(np.float32)
    got = _gpu_warp_grads(c, cuda_device, alpha=alpha)
    exact = _f64_warp_grads(c, alpha=alpha)
    fp32 = _f64_warp_grads(c, alpha=alpha, dtype=torch.float32)
    for key, v in got.items():
        assert_close_grad(v, exact[key], what=f"d_{key}", ref32=[fp32[key]])


def test_warp_positions_refuses_grad_inputs(cuda_device):
    """warp_positions stays forward-only: inputs that require grad under grad
    mode raise instead of silently cutting the graph."""
    from oss_b200 import warp_positions

    xy = torch.rand(4, 2, device=cuda_device, requires_grad=True)
    with pytest.raises(RuntimeError, match="forward-only"):
        warp_positions(xy, torch.zeros(2, 16, 16, device=cuda_device), (16, 16))


@torch.no_grad()
@pytest.mark.parametrize("alpha", [1.0, 0.5])
def test_warp_parked_renders_as_compacted(cuda_device, alpha):
    """warp_canvas(compact=False) keeps every slot: the survivors' values at
    their own slots equal the compacted ones bit for bit, the dropped slots are
    parked with zero opacity and colours, and a render of the parked canvas is
    the render of the compacted canvas bit for bit (the survivors keep their
    relative order in every tile list; a parked Gaussian bins into no tile)."""
    from oss_b200 import CanvasState, warp_canvas
    from oss_cuda import rasterize_gaussians

    n, h, w, hl, wl = 60_000, 270, 480, 135, 240
    rng = np.random.default_rng(41)
    pos = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    sc = np.exp(rng.standard_normal((n, 2)) * 0.3 + math.log(2.0)).astype(np.float32)
    rt = (rng.random(n) * math.pi).astype(np.float32)
    op = (1 / (1 + np.exp(-rng.standard_normal(n)))).astype(np.float32)
    col = rng.random((n, 3)).astype(np.float32)
    motion = smooth_motion(hl, wl, seed=42, max_mag=24.0)
    t = lambda a: torch.from_numpy(a).to(cuda_device)
    canvas = CanvasState(t(pos), t(sc), t(rt), t(op), t(col), n)
    packed = warp_canvas(canvas, t(motion[None]), (h, w), 0.5, alpha)
    parked = warp_canvas(canvas, t(motion[None]), (h, w), 0.5, alpha, compact=False)
    assert parked.count == n and 0 < packed.count < n
    keep = (parked.opacities != 0) | (parked.positions[:, 0] > -1.0e6)
    assert int(keep.sum()) == packed.count
    for a, b in ((parked.positions, packed.positions), (parked.scales, packed.scales),
                 (parked.rotations, packed.rotations), (parked.opacities, packed.opacities),
                 (parked.colors, packed.colors)):
        assert torch.equal(a[keep], b)
    assert not parked.opacities[~keep].any() and not parked.colors[~keep].any()
    for binning in ("tight3sigma", "exact56"):
        imgs = [rasterize_gaussians(c.positions, c.scales, c.rotations, c.colors, h, w, binning=binning,
                                    opacity=c.opacities) for c in (packed, parked)]
        assert torch.equal(imgs[0], imgs[1]), binning


def test_warp_parked_is_forward_only(cuda_device):
    from oss_b200 import CanvasState, warp_canvas

    n = 64
    pos = torch.rand((n, 2), device=cuda_device) * 32
    canvas = CanvasState(pos.requires_grad_(True), torch.ones((n, 2), device=cuda_device),
                         torch.zeros(n, device=cuda_device), torch.ones(n, device=cuda_device),
                         torch.ones((n, 3), device=cuda_device), n)
    with pytest.raises(RuntimeError, match="forward-only"):
        warp_canvas(canvas, torch.zeros((1, 2, 16, 16), device=cuda_device), (32, 32), compact=False)
