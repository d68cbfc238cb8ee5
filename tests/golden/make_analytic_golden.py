"""Golden vectors of the Analytic-Splatting pixel integral from the reference's
own code (oss/sr/v6/aa_analytic_splat.py: analytic_pixel_integral, logistic_cdf,
and their autograd).

Runs only where the reference tree is importable (OSS_REFERENCE_ROOT, as for
make_golden.py); writes the committed fixture analytic_cases.npz.

    OSS_REFERENCE_ROOT=/path/to/open-supersampling python tests/golden/make_analytic_golden.py

Cases: random anisotropic inverse covariances, diagonal ones, exactly isotropic
ones (the reference's isotropic branch), near-isotropic ones on both sides of
its 1e-5 eigengap test, very wide and very narrow Gaussians, non-symmetric
inputs; per-pixel offsets broadcast against per-Gaussian matrices.  Each stores
the inputs, the values and the gradients of sum(value * upstream) with respect
to delta_x, delta_y and sigma_2d_inv.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "analytic_cases.npz"


def main() -> None:
    root = os.environ.get("OSS_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set OSS_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, str(Path(root)))
    from oss.sr.v6.aa_analytic_splat import analytic_pixel_integral, logistic_cdf

    g = torch.Generator().manual_seed(0xA5)
    out = {}
    G, P = 64, 48
    # per-Gaussian inverse covariances
    th = torch.rand(G, generator=g) * 3.1
    s1 = torch.exp(torch.randn(G, generator=g) * 0.8)
    s2 = torch.exp(torch.randn(G, generator=g) * 0.8)
    c, s = torch.cos(th), torch.sin(th)
    R = torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2)
    Sig = R @ torch.diag_embed(torch.stack([s1 * s1, s2 * s2], -1)) @ R.transpose(-1, -2)
    inv = torch.linalg.inv(Sig)
    inv[:6] = torch.diag_embed(torch.rand(6, 2, generator=g) + 0.2)              # diagonal
    inv[6:10] = torch.eye(2) * (torch.rand(4, 1, 1, generator=g) + 0.3)          # exactly isotropic
    base = torch.eye(2) * 0.7
    inv[10] = base + torch.tensor([[3e-6, 0.0], [0.0, 0.0]])                       # gap 3e-6 (< 1e-5)
    inv[11] = base + torch.tensor([[3e-5, 0.0], [0.0, 0.0]])                       # gap 3e-5 (> 1e-5)
    inv[12] = torch.tensor([[1e-4, 0.0], [0.0, 1e-4]]) + torch.tensor([[2e-4, 1e-5], [1e-5, 0.0]])  # very wide
    inv[13] = torch.tensor([[40.0, 5.0], [5.0, 30.0]])                              # very narrow
    inv[14] = torch.tensor([[1.2, 0.3], [0.1, 0.8]])                                # non-symmetric
    dx = (torch.rand(G, P, generator=g) - 0.5) * 12.0
    dy = (torch.rand(G, P, generator=g) - 0.5) * 12.0
    dx[:, 0] = 0.0
    dy[:, 0] = 0.0
    up = torch.randn(G, P, generator=g)
    leaves = [t.clone().requires_grad_(True) for t in (dx, dy, inv)]
    val = analytic_pixel_integral(leaves[0], leaves[1], leaves[2].unsqueeze(-3).expand(G, 1, 2, 2).squeeze(1))
    (val * up).sum().backward()
    out["grid_dx"], out["grid_dy"], out["grid_inv"], out["grid_up"] = dx.numpy(), dy.numpy(), inv.numpy(), up.numpy()
    out["grid_val"] = val.detach().numpy()
    out["grid_d_dx"], out["grid_d_dy"], out["grid_d_inv"] = (t.grad.numpy() for t in leaves)
    # one matrix per offset (no broadcast)
    M = 500
    th = torch.rand(M, generator=g) * 3.1
    a1 = torch.exp(torch.randn(M, generator=g))
    a2 = torch.exp(torch.randn(M, generator=g))
    c, s = torch.cos(th), torch.sin(th)
    R = torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2)
    inv2 = R @ torch.diag_embed(torch.stack([a1, a2], -1)) @ R.transpose(-1, -2)
    dx2 = torch.randn(M, generator=g) * 2.0
    dy2 = torch.randn(M, generator=g) * 2.0
    up2 = torch.randn(M, generator=g)
    leaves = [t.clone().requires_grad_(True) for t in (dx2, dy2, inv2)]
    val2 = analytic_pixel_integral(*leaves)
    (val2 * up2).sum().backward()
    out["flat_dx"], out["flat_dy"], out["flat_inv"], out["flat_up"] = dx2.numpy(), dy2.numpy(), inv2.numpy(), up2.numpy()
    out["flat_val"] = val2.detach().numpy()
    out["flat_d_dx"], out["flat_d_dy"], out["flat_d_inv"] = (t.grad.numpy() for t in leaves)
    x = torch.linspace(-8, 8, 161)
    out["cdf_x"], out["cdf_val"] = x.numpy(), logistic_cdf(x).numpy()
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({len(out)} arrays)")


if __name__ == "__main__":
    main()
