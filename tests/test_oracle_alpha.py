"""The alpha-blend oracle (oracle/oss_oracle.c) against an independent float64
PyTorch restatement of the same compositing contract, differentiated by
autograd.  The reference has no alpha blending (its rasterizer is additive),
so this mode's parity is unpinned; these tests pin the oracle to the
contract's mathematics instead:
  a_i = min(0.99, opacity_i exp(-q_i/2)), skip a_i < 1/255, stop before the
  entry that would take T below 1e-4, C += feat a T, T *= 1 - a, out = C + T bg.
CPU only.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as orc


def scene(n, h, w, seed, dense=False):
    rng = np.random.default_rng(seed)
    if dense:
        xy = (np.array([w, h]) / 2 + (rng.random((n, 2)) - 0.5) * np.array([w, h]) * 0.6).astype(np.float32)
    else:
        xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    scale = (rng.random((n, 2)) * 4.0 + 1.0).astype(np.float32)
    rot = (rng.random(n) * 3.1).astype(np.float32)
    feat = rng.random((n, 3)).astype(np.float32)
    op = (rng.random(n) * 0.95 + 0.03).astype(np.float32)
    depth = rng.random(n).astype(np.float32)
    grad = rng.standard_normal((3, h, w)).astype(np.float32)
    return xy, scale, rot, feat, op, depth, grad


def torch_alpha(xy, conic, feat, op, gid, offs, h, w, bg):
    """Float64 compositing over the oracle's lists; decisions from the same fp32
    q and exp the oracle uses, values differentiable in float64."""
    ntx = (w + 15) // 16
    f = feat.shape[1]
    img = torch.zeros((f, h, w), dtype=torch.float64)
    k32 = conic.detach().float()
    xy32 = xy.detach().float()
    for t in range(offs.size - 1):
        b, e = int(offs[t]), int(offs[t + 1])
        tx0, ty0 = (t % ntx) * 16, (t // ntx) * 16
        ys, xs = torch.meshgrid(torch.arange(ty0, min(ty0 + 16, h)), torch.arange(tx0, min(tx0 + 16, w)),
                                indexing="ij")
        px, py = xs.reshape(-1).double(), ys.reshape(-1).double()
        T = torch.ones(px.numel(), dtype=torch.float64)
        C = torch.zeros((f, px.numel()), dtype=torch.float64)
        done = torch.zeros(px.numel(), dtype=torch.bool)
        for j in range(b, e):
            g = int(gid[j])
            dx32 = px.float() - xy32[g, 0]
            dy32 = py.float() - xy32[g, 1]
            q32 = k32[g, 0] * dx32 * dx32 + 2.0 * k32[g, 1] * dx32 * dy32 + k32[g, 2] * dy32 * dy32
            og_dec = op[g].detach().double() * torch.exp(-0.5 * q32).double()
            a_dec = torch.clamp(og_dec, max=0.99)
            valid = torch.isfinite(q32) & (q32 >= 0) & (a_dec >= 1.0 / 255.0) & ~done
            dx = px - xy[g, 0]
            dy = py - xy[g, 1]
            q = conic[g, 0] * dx * dx + 2.0 * conic[g, 1] * dx * dy + conic[g, 2] * dy * dy
            og = op[g] * torch.exp(-0.5 * q)
            a = torch.where(og_dec < 0.99, og, torch.full_like(og, 0.99))
            tn = T * (1.0 - a)
            stop = valid & (tn.detach() < 1e-4)
            done = done | stop
            valid = valid & ~stop
            C = C + torch.where(valid, feat[g][:, None] * a * T, torch.zeros_like(C))
            T = torch.where(valid, tn, T)
        out = C + T[None, :] * bg[:, None]
        img[:, ys.reshape(-1), xs.reshape(-1)] = out
    return img


@pytest.mark.parametrize("n,h,w,seed,dense", [(24, 32, 48, 1, False), (60, 48, 48, 2, True), (120, 40, 56, 3, True)])
def test_alpha_oracle_matches_float64_autograd(n, h, w, seed, dense):
    xy, scale, rot, feat, op, depth, grad = scene(n, h, w, seed, dense)
    bg = np.array([0.2, 0.0, 0.7], np.float32)
    conic, gid, offs = orc.alpha_lists(xy, scale, rot, depth, h, w)
    img, tf, nc, amb = orc.render_alpha_forward(xy, conic, feat, op, gid, offs, h, w, bg)
    # both sides decide from the same fp32 q and exp, so pixels near a threshold agree too;
    # the flag only matters against the GPU's exp2
    assert amb.mean() < 0.01
    leaves = [torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (xy, conic, feat, op)]
    ref = torch_alpha(*leaves, gid, offs, h, w, torch.tensor(bg, dtype=torch.float64))
    np.testing.assert_allclose(img, ref.detach().numpy(), rtol=1e-5, atol=1e-6)
    (ref * torch.tensor(grad, dtype=torch.float64)).sum().backward()
    d_xy, d_conic, d_feat, d_op = orc.render_alpha_backward(xy, conic, feat, op, gid, offs, grad, h, w, bg)
    for got, leaf, name in ((d_xy, leaves[0], "d_xy"), (d_conic, leaves[1], "d_conic"), (d_feat, leaves[2], "d_feat"),
                            (d_op, leaves[3], "d_opacity")):
        want = leaf.grad.numpy()
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5 * max(1.0, np.abs(want).max()), err_msg=name)
    assert (nc > 0).any() and (tf < 1.0).any()


def test_alpha_oracle_early_stop_and_contrib_counts():
    # 30 Gaussians of opacity 0.98 stacked on one pixel: T = 1 -> 0.02 -> 4e-4, the third
    # layer would take it to 8e-6 < 1e-4, so two composite
    n, h, w = 30, 16, 16
    xy = np.full((n, 2), 8.0, np.float32)
    scale = np.full((n, 2), 6.0, np.float32)
    rot = np.zeros(n, np.float32)
    feat = np.tile(np.array([[1.0, 0.5, 0.25]], np.float32), (n, 1))
    op = np.full(n, 0.98, np.float32)
    img, tf, nc, amb = orc.render_alpha(xy, scale, rot, feat, op, h, w, depth=np.arange(n, dtype=np.float32))
    a = np.float64(np.float32(0.98))
    assert nc[8, 8] == 2 and not amb[8, 8]
    np.testing.assert_allclose(tf[8, 8], (1 - a) ** 2, rtol=1e-6)
    np.testing.assert_allclose(img[:, 8, 8], feat[0] * (a + a * (1 - a)), rtol=1e-6)


def test_alpha_oracle_depth_order():
    rng = np.random.default_rng(5)
    n, h, w = 50, 32, 32
    xy = (rng.random((n, 2)) * 32).astype(np.float32)
    scale = (rng.random((n, 2)) * 3 + 1).astype(np.float32)
    rot = (rng.random(n) * 3).astype(np.float32)
    depth = rng.integers(0, 5, n).astype(np.float32)  # many ties: broken by gid
    depth[3] = -0.0
    conic, gid, offs = orc.alpha_lists(xy, scale, rot, depth, h, w)
    for t in range(offs.size - 1):
        seg = gid[offs[t]:offs[t + 1]]
        keys = list(zip((depth[seg] + 0.0).tolist(), seg.tolist()))
        assert keys == sorted(keys)
