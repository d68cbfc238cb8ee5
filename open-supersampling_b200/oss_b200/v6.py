"""v6 active-mask-aware feature rasterizer on the B200 kernels.

Drop-in for oss/sr/v6/rasterizer.py:17-345 (``V6Rasterizer``): the same
constructor arguments, ``forward(canvas, active_mask, output_hw,
return_weight_sum)`` contract, sanitisation rules, weight-sum channel, the
4-phase feathered overlap render and the batch expand.  Every render goes
through ``oss_cuda.rasterize_gaussians`` (liboss_b200.so), the feathered
overlap in one pass; the masking, sanitising and ones channel are one kernel
(oss_v6_sanitize) that keeps every live Gaussian's slot, so no survivor count
is read on the host.

``spawn_offset`` shifts all means by a per-frame integer
offset before rendering, the effect of the spawner offset of
oss/sr/v6/model.py:795-820 on the rasterized canvas.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn
from torch.autograd import Function

from oss_cuda import _lib, rasterize_gaussians
from oss_cuda._raster import stream_of
from oss_cuda.overlap import cosine_ramp, phase_feather_mask, render_overlapped_with  # noqa: F401

TILE_SIZE = 16
_MIN_PIXEL_SCALE = 1.0e-3


def render(xy, scale, rot, feat, h, w, binning=None, opacity=None):
    """One render through the native op, with the scale floor the reference's
    oss_cuda backend applies before calling it (rasterizer.py:186-195)."""
    return rasterize_gaussians(xy, scale.clamp_min(_MIN_PIXEL_SCALE), rot, feat, h, w, TILE_SIZE, True,
                               binning=binning, opacity=opacity)


def render_overlapped(xy, scale, rot, feat, h, w, overlap, binning=None, opacity=None):
    """Feathered overlapping-tile render (rasterizer.py:159-210): the blend of four
    renders whose 16-px tile grids are shifted by (0|-o, 0|-o), each cropped back
    to (h, w), weighted by its feather mask and normalised by the mask sum --
    computed in one pass by rasterize_gaussians(overlap=o) (csrc/feather.cu),
    with the scale floor of the reference's oss_cuda backend."""
    return rasterize_gaussians(xy, scale.clamp_min(_MIN_PIXEL_SCALE), rot, feat, h, w, TILE_SIZE, True,
                               binning=binning, opacity=opacity, overlap=overlap)


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.to(dtype=torch.float32).contiguous()


class _V6Sanitize(Function):
    """oss_v6_sanitize and its backward: the live canvas tensors -> the render's
    inputs (xy, scale, rot, feat with the optional ones channel), dropped
    Gaussians parked outside the frame."""

    @staticmethod
    def forward(ctx, pos, scl, rot, colors, mask, h, w, f_out, ones):
        n, f_in = int(pos.shape[0]), int(colors.shape[1])
        dev = pos.device
        f32 = dict(device=dev, dtype=torch.float32)
        xy, scale, r = torch.empty((n, 2), **f32), torch.empty((n, 2), **f32), torch.empty((n,), **f32)
        feat = torch.empty((n, f_out + (1 if ones else 0)), **f32)
        flags = torch.empty((n,), device=dev, dtype=torch.int16)
        lib = _lib.lib()
        with torch.cuda.device(dev):
            _lib.check(lib.oss_v6_sanitize(n, h, w, f_in, f_out, 1 if ones else 0, mask.data_ptr(), pos.data_ptr(),
                                           scl.data_ptr(), rot.data_ptr(), colors.data_ptr() if f_in else None,
                                           xy.data_ptr(), scale.data_ptr(), r.data_ptr(), feat.data_ptr(),
                                           flags.data_ptr(), stream_of(pos)), "oss_v6_sanitize")
        ctx.save_for_backward(flags)
        ctx.meta = (n, f_in, f_out, ones)
        return xy, scale, r, feat

    @staticmethod
    def backward(ctx, d_xy, d_scale, d_rot, d_feat):
        (flags,) = ctx.saved_tensors
        n, f_in, f_out, ones = ctx.meta
        dev = flags.device
        f32 = dict(device=dev, dtype=torch.float32)
        outs = [torch.empty((n, 2), **f32), torch.empty((n, 2), **f32), torch.empty((n,), **f32),
                torch.empty((n, f_in), **f32)]
        ins = [None if t is None else t.contiguous().float() for t in (d_xy, d_scale, d_rot, d_feat)]
        lib = _lib.lib()
        with torch.cuda.device(dev):
            _lib.check(lib.oss_v6_sanitize_backward(n, f_in, f_out, 1 if ones else 0, flags.data_ptr(),
                                                    *(None if t is None else t.data_ptr() for t in ins),
                                                    *(t.data_ptr() if t.numel() else None for t in outs),
                                                    stream_of(flags)), "oss_v6_sanitize_backward")
        return (*outs, None, None, None, None, None)


class V6Rasterizer(nn.Module):
    """Renders the active subset of a v6 canvas to an HR feature image.

    Same arguments as the reference class plus ``binning`` (list mode of the
    native op; the default reproduces the reference's full-tail sum).
    """

    def __init__(self, token_dim: int, latent_rank: int = 64, tile_size: int = TILE_SIZE, overlap: int = 0,
                 binning: str | None = None) -> None:
        super().__init__()
        if token_dim <= 0:
            raise ValueError(f"token_dim must be positive; got {token_dim}")
        if latent_rank <= 0:
            raise ValueError(f"latent_rank must be positive; got {latent_rank}")
        if tile_size != TILE_SIZE:
            raise ValueError(f"tile_size must match the underlying renderer ({TILE_SIZE}); got {tile_size}")
        if overlap < 0:
            raise ValueError(f"overlap must be >= 0; got {overlap}")
        self.token_dim = int(token_dim)
        self.latent_rank = int(latent_rank)
        self.feature_dim = self.latent_rank if self.latent_rank < 64 else self.token_dim
        self.tile_size = int(tile_size)
        self.overlap = int(overlap)
        self.binning = binning

    def forward(self, canvas, active_mask: torch.Tensor, output_hw: Tuple[int, int],
                return_weight_sum: bool | None = None, spawn_offset: torch.Tensor | None = None):
        if return_weight_sum is None:
            return_weight_sum = self.latent_rank < 64
        h, w = int(output_hw[0]), int(output_hw[1])
        if h <= 0 or w <= 0:
            raise ValueError(f"output_hw must be positive; got {output_hw}")
        batch, mask = self._normalize_active_mask(canvas, active_mask)
        device, out_dtype = canvas.colors.device, canvas.colors.dtype

        def zeros():
            feats = torch.zeros((batch, self.feature_dim, h, w), device=device, dtype=out_dtype)
            if return_weight_sum:
                return feats, torch.zeros((batch, 1, h, w), device=device, dtype=out_dtype)
            return feats

        n_live = max(0, min(int(canvas.count), int(canvas.positions.shape[0])))
        if n_live == 0:
            return zeros()
        colors = canvas.colors[:n_live]
        if colors.ndim != 2:
            raise ValueError(f"canvas.colors must be (N, F); got {tuple(colors.shape)}")
        feat_dtype = colors.dtype
        # the sanitisation and the ones channel on the device: every live Gaussian keeps
        # its slot (a dropped one bins into no tile), so no count is read on the host
        pos, scl, rot, feat = _V6Sanitize.apply(
            _f32(canvas.positions[:n_live]), _f32(canvas.scales[:n_live]), _f32(canvas.rotations[:n_live]),
            _f32(colors), mask[:n_live].to(device=device, dtype=torch.bool).contiguous(), h, w, self.feature_dim,
            bool(return_weight_sum))
        if spawn_offset is not None:
            pos = pos + spawn_offset.to(device=device, dtype=torch.float32).view(1, 2)
        if self.overlap > 0:
            img = render_overlapped(pos, scl, rot, feat, h, w, self.overlap, self.binning)
        else:
            img = render(pos, scl, rot, feat, h, w, self.binning)
        img = img.to(dtype=feat_dtype)
        feats = img[: self.feature_dim].unsqueeze(0).expand(batch, -1, -1, -1)
        if return_weight_sum:
            return feats, img[self.feature_dim: self.feature_dim + 1].unsqueeze(0).expand(batch, -1, -1, -1)
        return feats

    @staticmethod
    def _normalize_active_mask(canvas, active_mask: torch.Tensor):
        n = canvas.positions.shape[0]
        if active_mask.device != canvas.positions.device:
            active_mask = active_mask.to(device=canvas.positions.device)
        if active_mask.ndim == 1:
            if active_mask.shape[0] != n:
                raise ValueError(f"active_mask must have length {n}; got {active_mask.shape[0]}")
            return 1, active_mask.to(dtype=torch.bool)
        if active_mask.ndim == 2:
            b, m = active_mask.shape
            if m != n:
                raise ValueError(f"active_mask must have trailing length {n}; got {m}")
            mask = active_mask.to(dtype=torch.bool)
            if b == 0:
                raise ValueError("active_mask batch dimension must be positive")
            if b > 1 and not torch.equal(mask, mask[:1].expand_as(mask)):
                raise ValueError("batched active_mask rows must be identical because v6 renders the shared "
                                 "per-rank canvas once and expands it across B")
            return int(b), mask[0]
        raise ValueError(f"active_mask must be (N,) or (B, N); got {tuple(active_mask.shape)}")

    def _token_features(self, colors: torch.Tensor) -> torch.Tensor:
        if colors.ndim != 2:
            raise ValueError(f"canvas.colors must be (N, F); got {tuple(colors.shape)}")
        f = self.feature_dim
        if colors.shape[-1] == f:
            return colors
        if colors.shape[-1] > f:
            return colors[..., :f]
        return torch.nn.functional.pad(colors, (0, f - colors.shape[-1]))


def render_canvas_at_lr(rasterizer: V6Rasterizer, warped_canvas, active_mask, batch_size: int, h_lr: int,
                        w_lr: int, scale: float, device, dtype):
    """(G, m) for ConcatFusion (oss/sr/v6/model.py:628-678, ``_rasterize_canvas_at_lr``):
    the warped canvas, whose positions and scales live in HR pixels, divided by
    the upscale factor and rendered at LR resolution with the weight-sum channel.
    G is (B, latent_rank, h_lr, w_lr), m is (B, 1, h_lr, w_lr); both are zeros
    without a canvas.  ``active_mask`` None means every one of the canvas's
    ``count`` Gaussians."""
    from .canvas import CanvasState

    r = int(rasterizer.latent_rank)
    if warped_canvas is None or warped_canvas.count == 0:
        return (torch.zeros((batch_size, r, h_lr, w_lr), device=device, dtype=dtype),
                torch.zeros((batch_size, 1, h_lr, w_lr), device=device, dtype=dtype))
    scaled = CanvasState(positions=warped_canvas.positions / float(scale),
                         scales=warped_canvas.scales / float(scale), rotations=warped_canvas.rotations,
                         opacities=warped_canvas.opacities, colors=warped_canvas.colors, count=warped_canvas.count)
    mask = active_mask if active_mask is not None else torch.ones(int(warped_canvas.count), device=device,
                                                                  dtype=torch.bool)
    out = rasterizer(scaled, mask.unsqueeze(0).expand(batch_size, -1) if mask.ndim == 1 else mask,
                     output_hw=(h_lr, w_lr), return_weight_sum=True)
    if isinstance(out, tuple):
        g, m = out
    else:
        g = out
        m = torch.zeros((batch_size, 1, h_lr, w_lr), device=device, dtype=dtype)
    return g.to(dtype=dtype), m.to(dtype=dtype)
