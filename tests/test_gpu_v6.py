"""GPU V6 front-end (active mask, sanitisation, weight sum, feathered overlap)
against golden vectors of the reference's V6Rasterizer and _render_overlapped."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_close, assert_close_grad, golden_case, load_golden

pytestmark = pytest.mark.gpu


def test_v6_rasterizer_matches_reference(cuda_device):
    from oss_b200 import CanvasState, V6Rasterizer

    data = load_golden("v6_cases.npz")
    for name in data["names"]:
        c = golden_case(data, str(name))
        count, h, w, f, rank, ov, rws = (int(v) for v in c["meta"])
        leaves = [torch.from_numpy(c[k]).to(cuda_device).requires_grad_(True)
                  for k in ("positions", "scales", "rotations", "colors")]
        canvas = CanvasState(leaves[0], leaves[1], leaves[2], torch.from_numpy(c["opacities"]).to(cuda_device),
                             leaves[3], count)
        r = V6Rasterizer(token_dim=f, latent_rank=rank, overlap=ov)
        res = r(canvas, torch.from_numpy(c["mask"]).to(cuda_device), output_hw=(h, w),
                return_weight_sum=None if rws < 0 else bool(rws))
        feats, wsum = res if isinstance(res, tuple) else (res, None)
        assert_close(feats.detach().cpu().numpy(), c["feats"], what=f"{name} feats")
        loss = (feats[0] * torch.from_numpy(c["wf"]).to(cuda_device)).sum()
        if "wsum" in c:
            assert wsum is not None
            assert_close(wsum.detach().cpu().numpy(), c["wsum"], what=f"{name} weight sum")
            loss = loss + (wsum[0] * torch.from_numpy(c["ww"]).to(cuda_device)).sum()
        else:
            assert wsum is None
        loss.backward()
        for k, t in zip(("positions", "scales", "rotations", "colors"), leaves):
            assert_close_grad(t.grad.cpu().numpy(), c[f"d_{k}"], what=f"{name} d_{k}")


def test_render_overlapped_matches_reference(cuda_device):
    from oss_b200 import render_overlapped

    data = load_golden("overlap_cases.npz")
    for name in data["names"]:
        c = golden_case(data, str(name))
        h, w = (int(v) for v in c["hw"])
        leaves = [torch.from_numpy(c[k]).to(cuda_device).requires_grad_(True) for k in ("xy", "scale", "rot", "feat")]
        img = render_overlapped(*leaves, h, w, int(c["overlap"]))
        assert_close(img.detach().cpu().numpy(), c["image"], what=f"{name} image")
        img.backward(torch.from_numpy(c["grad"]).to(cuda_device))
        for k, t in zip(("xy", "scale", "rot", "feat"), leaves):
            assert_close_grad(t.grad.cpu().numpy(), c[f"d_{k}"], what=f"{name} d_{k}")


def test_v6_empty_and_spawn_offset(cuda_device):
    from oss_b200 import CanvasState, V6Rasterizer

    n = 10
    canvas = CanvasState(torch.rand(n, 2, device=cuda_device) * 32, torch.ones(n, 2, device=cuda_device),
                         torch.zeros(n, device=cuda_device), torch.ones(n, device=cuda_device),
                         torch.rand(n, 4, device=cuda_device), 0)
    r = V6Rasterizer(token_dim=4, latent_rank=2)
    feats, wsum = r(canvas, torch.ones(n, dtype=torch.bool, device=cuda_device), (32, 32))
    assert feats.shape == (1, 2, 32, 32) and float(feats.abs().sum()) == 0.0 and wsum.shape == (1, 1, 32, 32)
    canvas.count = n
    base = r(canvas, torch.ones(2, n, dtype=torch.bool, device=cuda_device), (64, 64), return_weight_sum=False)
    shifted = r(canvas, torch.ones(2, n, dtype=torch.bool, device=cuda_device), (64, 64), return_weight_sum=False,
                spawn_offset=torch.tensor([16.0, 16.0]))
    assert base.shape == (2, 2, 64, 64)
    # an integer 16-px shift moves the image by whole tiles: same pixels, shifted
    assert torch.allclose(shifted[0, :, 16:, 16:], base[0, :, :48, :48], atol=1e-5)


def test_v6_front_end_has_no_host_sync(cuda_device):
    """The sanitisation runs on the device (oss_v6_sanitize): V6Rasterizer.forward
    makes no synchronising torch call (the reference reads the active and
    surviving counts with .item()); dropped Gaussians -- inactive, non-finite,
    off the frame -- leave the image and every gradient untouched."""
    from oss_b200 import CanvasState, V6Rasterizer

    g = torch.Generator(device="cpu").manual_seed(5)
    n, h, w = 64, 48, 64
    pos = (torch.rand(n, 2, generator=g) * torch.tensor([w + 40.0, h + 40.0]) - 20.0).to(cuda_device)
    scl = (torch.rand(n, 2, generator=g) * 3.0 - 0.5).to(cuda_device)  # some negative, some below the floor
    rot = (torch.rand(n, generator=g) * 20.0 - 10.0).to(cuda_device)   # wrapped
    col = torch.rand(n, 5, generator=g).to(cuda_device)
    pos[3, 0] = float("nan")
    scl[4, 1] = float("inf")
    mask = torch.rand(n, generator=g).to(cuda_device) > 0.2
    leaves = [t.clone().requires_grad_(True) for t in (pos, scl, rot, col)]
    canvas = CanvasState(leaves[0], leaves[1], leaves[2], torch.ones(n, device=cuda_device), leaves[3], n)
    r = V6Rasterizer(token_dim=5, latent_rank=4)
    r(canvas, mask, (h, w))  # warm-up (library load, allocator)
    torch.cuda.synchronize()
    prev = torch.cuda.get_sync_debug_mode()
    torch.cuda.set_sync_debug_mode("error")
    try:
        sanitized = _v6_inputs(r, canvas, mask, h, w)
    finally:
        torch.cuda.set_sync_debug_mode(prev)
    feats, wsum = r(canvas, mask, (h, w))
    (feats.sum() + 2.0 * wsum.sum()).backward()
    keep = sanitized[4]
    assert not bool(keep[3]) and not bool(keep[4])
    assert not bool(keep[~mask].any())
    for t in leaves:
        assert torch.isfinite(t.grad).all()
        assert float(t.grad[~keep].abs().sum()) == 0.0
    # the kept ones: the reference's own eager sanitisation, restated, renders the same image
    kp = keep.nonzero().squeeze(1)
    xs = pos[kp].clamp_min(0.0)
    xs = torch.minimum(xs, torch.tensor([w - 1e-4, h - 1e-4], device=cuda_device))
    ss = scl[kp].abs().clamp(1e-3, float(max(h, w)))
    rs = torch.atan2(torch.sin(rot[kp]), torch.cos(rot[kp]))
    fs = torch.cat([col[kp, :4], torch.ones(kp.numel(), 1, device=cuda_device)], 1)
    from oss_cuda import rasterize_gaussians

    ref = rasterize_gaussians(xs, ss.clamp_min(1e-3), rs, fs, h, w)
    assert_close(feats[0].detach().cpu().numpy(), ref[:4].cpu().numpy(), what="kept-only render")
    assert_close(wsum[0].detach().cpu().numpy(), ref[4:5].cpu().numpy(), what="kept-only weight sum")


def _v6_inputs(r, canvas, mask, h, w):
    """The sanitised render inputs V6Rasterizer builds (xy, scale, rot, feat, kept)."""
    from oss_b200.v6 import _V6Sanitize, _f32

    n = int(canvas.count)
    xy, scale, rot, feat = _V6Sanitize.apply(_f32(canvas.positions[:n]), _f32(canvas.scales[:n]),
                                            _f32(canvas.rotations[:n]), _f32(canvas.colors[:n]),
                                            mask[:n].contiguous(), h, w, r.feature_dim, True)
    return xy, scale, rot, feat, xy[:, 0] > -1.0e6
