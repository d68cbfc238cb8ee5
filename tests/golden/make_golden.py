"""Generate golden vectors from the reference's own PyTorch implementation.

Runs only where the reference tree is importable (set OSS_REFERENCE_ROOT, e.g.
to a checkout of cashcon57/open-supersampling).  The outputs are small .npz
fixtures committed next to this script; tests read the fixtures, never the
reference tree.

    OSS_REFERENCE_ROOT=/path/to/open-supersampling python tests/golden/make_golden.py

Fixtures
  render_cases.npz   Rasterizer._render_reference (oss/gaussian/renderer/rasterizer.py:248-301)
                     forward images and autograd gradients (d_xy, d_scale, d_rot,
                     d_feat), plus d_conic through its conic= override (:253,263-290),
                     on the input distribution of tests/cuda/test_rasterizer_*_equivalence.py.
  tight_lists.npz    3-sigma tile lists built by the reference test's own list
                     construction (_ref_pair_construction, tests/cuda/
                     test_pair_construction_kernel.py:9-38) fed with the
                     tight-ellipse AABB of rasterizer_fwd.cu:74-108 evaluated in
                     torch fp32 (the formula of tests/perf/test_h008_tight_ellipse_aabb.py).
  warp_cases.npz     oss/sr/v6/canvas_warp.warp_canvas outputs (GS-STVSR warp) and
                     oss/gaussian/canvas/warp.warp_positions outputs.
  overlap_cases.npz  V6Rasterizer._render_overlapped (oss/sr/v6/rasterizer.py:159-210)
                     with overlap=4 over the reference backend.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
SEED = 0xC0DA


def _ref_root() -> Path:
    root = os.environ.get("OSS_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set OSS_REFERENCE_ROOT to the reference checkout")
    return Path(root)


def _inputs(n, h, w, f, seed):
    g = torch.Generator().manual_seed(seed)
    xy = torch.rand(n, 2, generator=g) * torch.tensor([float(w), float(h)])
    scale = torch.rand(n, 2, generator=g) * 5.0 + 0.5
    rot = torch.rand(n, generator=g) * 6.28
    feat = torch.randn(n, f, generator=g)
    grad = torch.randn(f, h, w, generator=g)
    return xy, scale, rot, feat, grad


def render_cases():
    from oss.gaussian.renderer.rasterizer import GaussianBatch, Rasterizer

    rast = Rasterizer(tile_size=16, topk_norm=True, force_backend="reference")
    cases = [("a", 16, 32, 32, 3), ("b", 64, 64, 128, 1), ("c", 24, 37, 53, 12), ("d", 1, 16, 16, 2),
             ("e", 48, 48, 80, 4)]
    out = {}
    for i, (name, n, h, w, f) in enumerate(cases):
        xy, scale, rot, feat, grad = _inputs(n, h, w, f, SEED + i)
        leaves = [t.clone().requires_grad_(True) for t in (xy, scale, rot, feat)]
        img = rast._render_reference(GaussianBatch(*leaves), h, w)
        img.backward(grad)
        out[f"{name}_xy"], out[f"{name}_scale"], out[f"{name}_rot"], out[f"{name}_feat"] = (
            t.numpy() for t in (xy, scale, rot, feat))
        out[f"{name}_grad"] = grad.numpy()
        out[f"{name}_hw"] = np.array([h, w], np.int32)
        out[f"{name}_image"] = img.detach().numpy()
        for k, t in zip(("d_xy", "d_scale", "d_rot", "d_feat"), leaves):
            out[f"{name}_{k}"] = t.grad.numpy()
        # d_conic through the conic= override, conic from the reference formula
        from tests.cuda.test_rasterizer_backward_equivalence import _conic_from_scale_rot

        conic = _conic_from_scale_rot(scale, rot).clone().requires_grad_(True)
        img2 = rast._render_reference(GaussianBatch(xy, scale, rot, feat), h, w, conic=conic)
        img2.backward(grad)
        out[f"{name}_conic"] = conic.detach().numpy()
        out[f"{name}_d_conic"] = conic.grad.numpy()
    out["names"] = np.array([c[0] for c in cases])
    np.savez_compressed(OUT / "render_cases.npz", **out)


def _tight_preprocess(xy, scale, rot, H, W, tile_size=16):
    """Tight-ellipse AABB (rasterizer_fwd.cu:74-108) in torch fp32."""
    from tests.cuda.test_preprocess_kernel import _ref_preprocess

    conic, _, _ = _ref_preprocess(xy, scale, rot, H, W, tile_size)
    a, b, d = conic[:, 0], conic[:, 1], conic[:, 2]
    det = a * d - b * b
    tau = torch.tensor(9.0)
    rx = torch.where(det > 1e-12, torch.sqrt(tau * d / det), 3.0 * torch.maximum(scale[:, 0], scale[:, 1]))
    ry = torch.where(det > 1e-12, torch.sqrt(tau * a / det), 3.0 * torch.maximum(scale[:, 0], scale[:, 1]))
    num_tx = (W + tile_size - 1) // tile_size
    num_ty = (H + tile_size - 1) // tile_size
    x_lo = ((xy[:, 0] - rx) / tile_size).floor().clamp_(0, num_tx).to(torch.int32)
    x_hi = ((xy[:, 0] + rx) / tile_size).ceil().clamp_(0, num_tx).to(torch.int32)
    y_lo = ((xy[:, 1] - ry) / tile_size).floor().clamp_(0, num_ty).to(torch.int32)
    y_hi = ((xy[:, 1] + ry) / tile_size).ceil().clamp_(0, num_ty).to(torch.int32)
    aabb = torch.stack([x_lo, y_lo, x_hi, y_hi], dim=-1)
    pair_count = ((x_hi - x_lo).clamp_min(0) * (y_hi - y_lo).clamp_min(0)).to(torch.int32)
    finite = a.isfinite() & b.isfinite() & d.isfinite()
    pair_count = torch.where(finite, pair_count, torch.zeros_like(pair_count))
    return conic, aabb, pair_count


def tight_lists():
    import tests.cuda.test_pair_construction_kernel as tpc

    tpc._ref_preprocess = _tight_preprocess  # the reference helper's list builder, tight AABBs
    cases = [("a", 4, 64, 64), ("b", 16, 64, 64), ("c", 64, 256, 256), ("d", 256, 270, 480), ("e", 200, 37, 91)]
    out = {}
    for i, (name, n, h, w) in enumerate(cases):
        torch.manual_seed(SEED + 100 + i)
        xy = torch.rand(n, 2) * torch.tensor([float(w), float(h)])
        scale = torch.rand(n, 2) * 5.0 + 0.5
        rot = torch.rand(n) * 6.28
        gid, offs, conic, total = tpc._ref_pair_construction(xy, scale, rot, h, w, 16)
        _, aabb, count = _tight_preprocess(xy, scale, rot, h, w, 16)
        out[f"{name}_xy"], out[f"{name}_scale"], out[f"{name}_rot"] = xy.numpy(), scale.numpy(), rot.numpy()
        out[f"{name}_hw"] = np.array([h, w], np.int32)
        out[f"{name}_gid"] = gid.numpy().astype(np.int32)
        out[f"{name}_offsets"] = offs.numpy().astype(np.int32)
        out[f"{name}_conic"] = conic.numpy()
        out[f"{name}_aabb"] = aabb.numpy()
        out[f"{name}_count"] = count.numpy()
    out["names"] = np.array([c[0] for c in cases])
    np.savez_compressed(OUT / "tight_lists.npz", **out)


def _smooth_motion(b, h, w, seed, max_mag):
    """Sum of 8 random sinusoids per channel, max |m| <= max_mag."""
    g = torch.Generator().manual_seed(seed)
    yy, xx = torch.meshgrid(torch.arange(h, dtype=torch.float64), torch.arange(w, dtype=torch.float64),
                            indexing="ij")
    out = torch.zeros(b, 2, h, w, dtype=torch.float64)
    for bi in range(b):
        for ch in range(2):
            amp = torch.rand(8, generator=g, dtype=torch.float64)
            fx = (torch.rand(8, generator=g, dtype=torch.float64) - 0.5) * (2.0 / 64.0)
            fy = (torch.rand(8, generator=g, dtype=torch.float64) - 0.5) * (2.0 / 64.0)
            ph = torch.rand(8, generator=g, dtype=torch.float64) * 2 * math.pi
            field = sum(amp[k] * torch.sin(2 * math.pi * (fx[k] * xx + fy[k] * yy) + ph[k]) for k in range(8))
            out[bi, ch] = field / amp.sum() * max_mag
    return out.to(torch.float32)


def warp_cases():
    from oss.gaussian.canvas.warp import warp_positions
    from oss.sr.v6.canvas_warp import warp_canvas
    from oss.sr.v6.model import CanvasState

    cases = [("a", 64, (16, 24), (32, 48), 1.0, 0.5), ("b", 96, (24, 40), (24, 40), 1.0, 0.5),
             ("c", 80, (18, 30), (36, 60), 0.5, 0.5), ("d", 50, (20, 20), (40, 40), 1.0, 0.25)]
    out = {}
    for i, (name, n, lr, hr, alpha, recon) in enumerate(cases):
        g = torch.Generator().manual_seed(SEED + 200 + i)
        h, w = hr
        pos = torch.rand(n, 2, generator=g) * torch.tensor([float(w), float(h)])
        scales = torch.exp(torch.randn(n, 2, generator=g) * 0.3 + math.log(1.5))
        rots = torch.rand(n, generator=g) * math.pi
        ops = torch.sigmoid(torch.randn(n, generator=g))
        cols = torch.rand(n, 3, generator=g)
        motion = _smooth_motion(2, lr[0], lr[1], SEED + 300 + i, max_mag=6.0)
        if name == "d":  # pure-scaling field (tests/sr/v6/test_canvas_warp.py:79-92 shape)
            yy, xx = torch.meshgrid(torch.arange(lr[0]), torch.arange(lr[1]), indexing="ij")
            motion[0, 0] = 0.5 * xx
            motion[0, 1] = 0.5 * yy
        canvas = CanvasState(positions=pos, scales=scales, rotations=rots, opacities=ops, colors=cols, count=n)
        res = warp_canvas(canvas, motion * alpha, output_hw=hr, sigma_recon=recon)
        out[f"{name}_positions"], out[f"{name}_scales"], out[f"{name}_rotations"] = pos.numpy(), scales.numpy(), rots.numpy()
        out[f"{name}_opacities"], out[f"{name}_colors"] = ops.numpy(), cols.numpy()
        out[f"{name}_motion"] = motion.numpy()
        out[f"{name}_hw"] = np.array(hr, np.int32)
        out[f"{name}_alpha"] = np.float32(alpha)
        out[f"{name}_recon"] = np.float32(recon)
        out[f"{name}_out_positions"] = res.positions.numpy()
        out[f"{name}_out_scales"] = res.scales.numpy()
        out[f"{name}_out_rotations"] = res.rotations.numpy()
        out[f"{name}_out_opacities"] = res.opacities.numpy()
        out[f"{name}_out_colors"] = res.colors.numpy()
        out[f"{name}_out_count"] = np.int32(res.count)
        # alpha-scaled position-only warp at HR (oss/gaussian/canvas/warp.py:28-91)
        m_hr = torch.nn.functional.interpolate(motion[:1], size=hr, mode="bilinear", align_corners=False)[0]
        new_xy, in_frame = warp_positions(pos, m_hr * float(alpha), hr)
        out[f"{name}_pw_motion_hr"] = m_hr.numpy()
        out[f"{name}_pw_xy"] = new_xy.numpy()
        out[f"{name}_pw_in_frame"] = in_frame.numpy()
    out["names"] = np.array([c[0] for c in cases])
    np.savez_compressed(OUT / "warp_cases.npz", **out)


def overlap_cases():
    from oss.gaussian.renderer.rasterizer import GaussianBatch
    from oss.sr.v6.rasterizer import V6Rasterizer

    cases = [("a", 12, 40, 56, 3, 4), ("b", 20, 33, 47, 4, 4)]
    out = {}
    for i, (name, n, h, w, f, ov) in enumerate(cases):
        xy, scale, rot, feat, grad = _inputs(n, h, w, f, SEED + 400 + i)
        r = V6Rasterizer(token_dim=f, overlap=ov)
        r.renderer.force_backend = "reference"
        leaves = [t.clone().requires_grad_(True) for t in (xy, scale, rot, feat)]
        img = r._render_overlapped(GaussianBatch(*leaves), output_hw=(h, w))
        img.backward(grad)
        out[f"{name}_xy"], out[f"{name}_scale"], out[f"{name}_rot"], out[f"{name}_feat"] = (
            t.numpy() for t in (xy, scale, rot, feat))
        out[f"{name}_grad"] = grad.numpy()
        out[f"{name}_hw"] = np.array([h, w], np.int32)
        out[f"{name}_overlap"] = np.int32(ov)
        out[f"{name}_image"] = img.detach().numpy()
        for k, t in zip(("d_xy", "d_scale", "d_rot", "d_feat"), leaves):
            out[f"{name}_{k}"] = t.grad.numpy()
    out["names"] = np.array([c[0] for c in cases])
    np.savez_compressed(OUT / "overlap_cases.npz", **out)


def v6_cases():
    """V6Rasterizer.forward (oss/sr/v6/rasterizer.py:56-157): active mask, live count,
    sanitisation (non-finite drop, |scale| clamp, frame-overlap cull, position clamp,
    rotation wrap), weight-sum channel, optional overlap, batch expand; plus gradients
    of a weighted sum of the outputs w.r.t. the canvas tensors."""
    from oss.sr.v6.model import CanvasState
    from oss.sr.v6.rasterizer import V6Rasterizer

    cases = [("a", 40, 48, 64, 8, 4, 0, True), ("b", 30, 40, 56, 3, 64, 4, None), ("c", 25, 33, 47, 5, 64, 0, False)]
    out = {}
    for i, (name, n, h, w, f, rank, ov, rws) in enumerate(cases):
        g = torch.Generator().manual_seed(SEED + 500 + i)
        pos = torch.rand(n, 2, generator=g) * torch.tensor([w * 1.3, h * 1.3]) - torch.tensor([w * 0.15, h * 0.15])
        scales = torch.rand(n, 2, generator=g) * 4.0 + 0.3
        scales[::7, 0] *= -1.0                      # negative scales are |.|-clamped
        scales[3, 1] = 1e-5                          # below the 1e-3 floor
        rots = torch.rand(n, generator=g) * 12.0 - 6.0
        cols = torch.randn(n, f, generator=g)
        ops = torch.rand(n, generator=g)
        pos[5, 0] = float("nan")                     # non-finite entries are dropped
        cols[6, 0] = float("inf")
        pos[8] = torch.tensor([-500.0, 10.0])        # far off-screen: culled
        count = n - 3                                # the last 3 entries are not live
        mask = torch.rand(n, generator=g) > 0.2
        leaves = [t.clone().requires_grad_(True) for t in (pos, scales, rots, cols)]
        canvas = CanvasState(positions=leaves[0], scales=leaves[1], rotations=leaves[2], opacities=ops,
                             colors=leaves[3], count=count)
        r = V6Rasterizer(token_dim=f, latent_rank=rank, overlap=ov)
        r.renderer.force_backend = "reference"
        res = r(canvas, mask, output_hw=(h, w), return_weight_sum=rws)
        feats, wsum = (res if isinstance(res, tuple) else (res, None))
        wf = torch.randn(feats.shape[1:], generator=g)
        loss = (feats[0] * wf).sum()
        if wsum is not None:
            ww = torch.randn(wsum.shape[1:], generator=g)
            loss = loss + (wsum[0] * ww).sum()
            out[f"{name}_ww"] = ww.numpy()
            out[f"{name}_wsum"] = wsum.detach().numpy()
        loss.backward()
        out[f"{name}_wf"] = wf.numpy()
        out[f"{name}_feats"] = feats.detach().numpy()
        for k, t in zip(("positions", "scales", "rotations", "colors"), leaves):
            out[f"{name}_{k}"] = t.detach().numpy()
            out[f"{name}_d_{k}"] = t.grad.numpy()
        out[f"{name}_opacities"] = ops.numpy()
        out[f"{name}_mask"] = mask.numpy()
        out[f"{name}_meta"] = np.array([count, h, w, f, rank, ov, -1 if rws is None else int(rws)], np.int64)
    out["names"] = np.array([c[0] for c in cases])
    np.savez_compressed(OUT / "v6_cases.npz", **out)


def main():
    root = _ref_root()
    sys.path.insert(0, str(root))
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    render_cases()
    tight_lists()
    warp_cases()
    overlap_cases()
    v6_cases()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
