"""Feathered overlapping-tile rendering (the reference's
``V6Rasterizer._render_overlapped``, oss/sr/v6/rasterizer.py:159-242), on any
render function with the ``rasterize_gaussians`` signature.

Four renders whose 16-px tile grids are shifted by (0|-o, 0|-o) are cropped
back to (h, w), weighted by a cosine ramp over the distance to the nearest
tile edge of their grid, and normalised by the weight sum, so no pixel sits
on a tile edge of every render.
"""
from __future__ import annotations

import math
from typing import Callable, Tuple

import torch

TILE_SIZE = 16

PHASES = ((0, 0), (-1, 0), (0, -1), (-1, -1))  # (dy, dx) multiples of the overlap


def cosine_ramp(t: torch.Tensor) -> torch.Tensor:
    return 0.5 - 0.5 * torch.cos(t * math.pi)


def phase_feather_mask(h: int, w: int, origin: Tuple[int, int], overlap: int, device) -> torch.Tensor:
    """Weight of one phase-shifted render: a cosine ramp over the distance to the
    nearest tile edge of that phase's grid (rasterizer.py:212-234)."""
    if overlap <= 0:
        return torch.ones((1, h, w), device=device, dtype=torch.float32)
    tile = float(TILE_SIZE)
    oy, ox = float(origin[0]), float(origin[1])
    py = torch.remainder(torch.arange(h, device=device, dtype=torch.float32) + 0.5 - oy, tile)
    px = torch.remainder(torch.arange(w, device=device, dtype=torch.float32) + 0.5 - ox, tile)
    wy = cosine_ramp((torch.minimum(py, tile - py) / float(overlap)).clamp(0.0, 1.0))
    wx = cosine_ramp((torch.minimum(px, tile - px) / float(overlap)).clamp(0.0, 1.0))
    return (wy.view(1, h, 1) * wx.view(1, 1, w)).to(torch.float32)


def render_overlapped_with(render: Callable, xy, scale, rot, feat, h: int, w: int, overlap: int):
    """The 4-phase feathered render through `render(xy, scale, rot, feat, h, w)`
    (differentiable whenever `render` is)."""
    device = xy.device
    f = int(feat.shape[1])
    accum = torch.zeros((f, h, w), device=device, dtype=torch.float32)
    wsum = torch.zeros((1, h, w), device=device, dtype=torch.float32)
    for py, px in PHASES:
        oy, ox = py * overlap, px * overlap
        crop_h = -(-(h - min(oy, 0)) // TILE_SIZE) * TILE_SIZE
        crop_w = -(-(w - min(ox, 0)) // TILE_SIZE) * TILE_SIZE
        shift = torch.tensor([float(ox), float(oy)], device=device, dtype=xy.dtype)
        img = render(xy - shift, scale, rot, feat, crop_h, crop_w)
        ys, xs = -min(oy, 0), -min(ox, 0)
        img = img[:, ys:ys + h, xs:xs + w]
        mask = phase_feather_mask(h, w, (oy, ox), overlap, device)
        accum = accum + img * mask
        wsum = wsum + mask
    return accum / wsum.clamp_min(1.0e-6)
