"""Golden vectors of the v7 N-D time-slice rasterizer from the reference's own
code (oss/sr/v7/nd_rasterizer.py: render_nd_time_slice and its autograd).

Runs only where the reference tree is importable (OSS_REFERENCE_ROOT, as for
make_golden.py); writes the committed fixture nd_cases.npz.

    OSS_REFERENCE_ROOT=/path/to/open-supersampling python tests/golden/make_nd_golden.py

Each case stores the inputs (means, covs, features, opacities, t_query, image
size, filter settings), the (R, H, W) image and the gradients of
sum(image * upstream) with respect to the four inputs.  Means are redrawn until
every cull-box bound (mean -+ 3 sqrt(largest eigenvalue)) lies at least 1e-3 px
from an integer, so the box is the same under any fp32 eigenvalue routine.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "nd_cases.npz"


def main() -> None:
    root = os.environ.get("OSS_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set OSS_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, str(Path(root)))
    from oss.sr.v7.nd_rasterizer import (_apply_2d_mip_filter, _apply_3d_smoothing_filter, render_nd_time_slice,
                                         time_marginal)

    g = torch.Generator().manual_seed(0x7D)
    out = {}
    cases = [("a", 60, 40, 56, 3, 0.4, True, 0.2, 0.1), ("b", 120, 48, 80, 8, 0.75, True, 0.2, 0.1),
             ("c", 40, 32, 48, 4, 0.1, False, 0.0, 0.0), ("d", 80, 36, 52, 40, 0.5, True, 0.3, 0.2)]
    for name, n, h, w, r, tq, falloff, v3, v2 in cases:
        for attempt in range(200):
            means = torch.rand(n, 3, generator=g) * torch.tensor([w + 8.0, h + 8.0, 1.0]) - torch.tensor(
                [4.0, 4.0, 0.0])
            L = torch.randn(n, 3, 3, generator=g) * torch.tensor([[1.6, 0.0, 0.0], [0.5, 1.4, 0.0],
                                                                  [0.3, 0.2, 0.25]])
            L = torch.tril(L)
            covs = L @ L.transpose(-1, -2) + torch.diag(torch.tensor([0.3, 0.3, 0.02]))
            opac = torch.rand(n, generator=g) * 0.9 + 0.05
            # cull-box margins of the reference's bounds
            cf, of = _apply_3d_smoothing_filter(covs, opac, v3)
            mc, cc, wt = time_marginal(means, cf, tq)
            cc, _ = _apply_2d_mip_filter(cc, wt, v2)
            lam = torch.linalg.eigvalsh(cc.float()).clamp(min=1e-6).amax(-1)
            rad = 3.0 * lam.sqrt().double()
            ends = torch.cat([mc.double() - rad[:, None], mc.double() + rad[:, None]], dim=-1)
            frac = (ends - ends.round()).abs()
            if bool((frac > 1e-3).all()):
                break
        else:
            raise SystemExit(f"no margin-safe draw for case {name}")
        feats = torch.rand(n, r, generator=g) * 2.0 - 0.5
        up = torch.randn(r, h, w, generator=g)
        leaves = [t.clone().requires_grad_(True) for t in (means, covs, feats, opac)]
        img = render_nd_time_slice(leaves[0], leaves[1], leaves[2], leaves[3], tq, (h, w), time_falloff=falloff,
                                   mip_3d_variance=v3, mip_2d_variance=v2)
        (img * up).sum().backward()
        out[f"{name}_means"], out[f"{name}_covs"] = means.numpy(), covs.numpy()
        out[f"{name}_feats"], out[f"{name}_opac"] = feats.numpy(), opac.numpy()
        out[f"{name}_up"], out[f"{name}_img"] = up.numpy(), img.detach().numpy()
        out[f"{name}_args"] = np.array([h, w, tq, float(falloff), v3, v2])
        for k, t in zip(("means", "covs", "feats", "opac"), leaves):
            out[f"{name}_d_{k}"] = t.grad.numpy()
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({len(out)} arrays)")


if __name__ == "__main__":
    main()
