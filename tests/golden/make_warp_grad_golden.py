"""Golden gradients of the reference's canvas warp (oss/sr/v6/canvas_warp.py:177-254
with covariance_resampling.py:76-116), taken by PyTorch autograd through the
reference's own code.

Runs only where the reference tree is importable (OSS_REFERENCE_ROOT, as
make_golden.py); writes warp_grad_cases.npz next to this script.

    OSS_REFERENCE_ROOT=/path/to/open-supersampling python tests/golden/make_warp_grad_golden.py

Each case holds the canvas and motion inputs, the upstream gradients of the
warped outputs (seeded, drawn after the forward since their row count is the
survivor count) and the reference's gradients of every input.  Case "flow" is
the setup of tests/sr/v6/test_canvas_warp.py:94-101 (three Gaussians of its
_canvas helper, zero motion 32x32 -> 64x64, loss = positions.sum()).
"""
from __future__ import annotations

import math
import sys

import numpy as np
import torch

from make_golden import OUT, SEED, _ref_root, _smooth_motion


def _case(name, n, lr, hr, recon, seed, motion=None, layout="random"):
    from oss.sr.v6.canvas_warp import warp_canvas
    from oss.sr.v6.model import CanvasState

    g = torch.Generator().manual_seed(seed)
    h, w = hr
    if layout == "flow":  # the reference test's _canvas(n) helper, tests/sr/v6/test_canvas_warp.py:10-33
        pos = torch.stack([torch.linspace(8.0, 32.0, n), torch.linspace(10.0, 34.0, n)], dim=-1)
        scales = torch.stack([torch.linspace(1.0, 1.6, n), torch.linspace(0.6, 1.2, n)], dim=-1)
        rots = torch.linspace(0.0, 0.3, n)
        ops = torch.linspace(0.2, 1.0, n)
        cols = torch.randn(n, 8, generator=g)
    else:  # means over the frame and a margin beyond it, so that some leave it
        pos = torch.rand(n, 2, generator=g) * torch.tensor([w + 6.0, h + 6.0]) - 3.0
        scales = torch.exp(torch.randn(n, 2, generator=g) * 0.4 + math.log(1.5))
        rots = torch.rand(n, generator=g) * math.pi
        ops = torch.sigmoid(torch.randn(n, generator=g))
        cols = torch.rand(n, 3, generator=g)
    if motion is None:
        motion = _smooth_motion(1, lr[0], lr[1], seed + 1, max_mag=4.0)
    leaves = [t.clone().requires_grad_(True) for t in (pos, scales, rots, ops, cols, motion)]
    canvas = CanvasState(positions=leaves[0], scales=leaves[1], rotations=leaves[2], opacities=leaves[3],
                         colors=leaves[4], count=n)
    res = warp_canvas(canvas, leaves[5], output_hw=hr, sigma_recon=recon)
    outs = (res.positions, res.scales, res.rotations, res.opacities, res.colors)
    if layout == "flow":
        ups = [torch.ones_like(outs[0])] + [torch.zeros_like(o) for o in outs[1:]]
    else:
        ups = [torch.randn(o.shape, generator=g) for o in outs]
    loss = sum((o * u).sum() for o, u in zip(outs, ups))
    loss.backward()
    out = {f"{name}_{k}": t.detach().numpy() for k, t in
           zip(("positions", "scales", "rotations", "opacities", "colors", "motion"), (pos, scales, rots, ops, cols,
                                                                                       motion))}
    for k, u in zip(("positions", "scales", "rotations", "opacities", "colors"), ups):
        out[f"{name}_g_{k}"] = u.numpy()
    for k, t in zip(("positions", "scales", "rotations", "opacities", "colors", "motion"), leaves):
        out[f"{name}_d_{k}"] = (t.grad if t.grad is not None else torch.zeros_like(t)).numpy()
    out[f"{name}_hw"] = np.array(hr, np.int32)
    out[f"{name}_recon"] = np.float32(recon)
    out[f"{name}_out_count"] = np.int32(res.count)
    return out


def warp_grad_cases():
    out = {}
    cases = [("a", 48, (12, 16), (24, 32), 0.25, SEED + 700),
             ("b", 64, (20, 28), (20, 28), 0.5, SEED + 701),
             ("c", 40, (10, 14), (30, 42), 0.5, SEED + 702)]
    for name, n, lr, hr, recon, seed in cases:
        out.update(_case(name, n, lr, hr, recon, seed))
    out.update(_case("flow", 3, (32, 32), (64, 64), 0.5, SEED + 703, motion=torch.zeros(1, 2, 32, 32),
                     layout="flow"))
    out["names"] = np.array([c[0] for c in cases] + ["flow"])
    np.savez_compressed(OUT / "warp_grad_cases.npz", **out)


if __name__ == "__main__":
    sys.path.insert(0, str(_ref_root()))
    warp_grad_cases()
    print("wrote", OUT / "warp_grad_cases.npz")
