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
