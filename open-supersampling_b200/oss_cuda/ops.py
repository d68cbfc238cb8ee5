"""Dispatcher-visible operators over the C ABI (torch.library custom ops).

The reference's op is a compiled extension module whose functions the
dispatcher sees (oss/cuda/src/bindings.cpp:65-78).  Here the kernels are
reached through ctypes, which torch.compile cannot trace; these registrations
make the additive render an opaque operator with a fake (shape-only) kernel
and an autograd formula, so that a compiled graph holds one node per render
instead of breaking around it:

  oss_b200::rasterize_sum           (xy, scale, rot, feat, opacity?, h, w, mode,
                                     capacity) -> image (F, H, W)
  oss_b200::rasterize_sum_backward  (..., grad_image) -> (d_xy, d_scale, d_rot,
                                     d_feat, d_opacity)

rasterize_gaussians routes through them while torch.compile traces it.  The
backward operator bins again (the saved tensors of an opaque operator cannot
have data-dependent sizes), so a compiled step bins twice; eager calls keep
the autograd Function that reuses the forward's lists and entry records.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _raster

_NAMESPACE = "oss_b200"


@torch.library.custom_op(f"{_NAMESPACE}::rasterize_sum", mutates_args=())
def rasterize_sum(xy: torch.Tensor, scale: torch.Tensor, rot: torch.Tensor, feat: torch.Tensor,
                  opacity: Optional[torch.Tensor], h: int, w: int, mode: int, capacity: int) -> torch.Tensor:
    with torch.cuda.device(xy.device):
        b = _raster.bin_gaussians(xy, scale, rot, h, w, mode, capacity=None if capacity < 0 else capacity,
                                  feat=feat, opacity=opacity)
        return _raster.render_forward(b, _raster.aligned(feat, 4), opacity)


@rasterize_sum.register_fake
def _rasterize_sum_fake(xy, scale, rot, feat, opacity, h, w, mode, capacity):
    return feat.new_empty((feat.shape[1], h, w))


@torch.library.custom_op(f"{_NAMESPACE}::rasterize_sum_backward", mutates_args=())
def rasterize_sum_backward(xy: torch.Tensor, scale: torch.Tensor, rot: torch.Tensor, feat: torch.Tensor,
                           opacity: Optional[torch.Tensor], grad: torch.Tensor, h: int, w: int, mode: int,
                           capacity: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                   torch.Tensor]:
    with torch.cuda.device(xy.device):
        b = _raster.bin_gaussians(xy, scale, rot, h, w, mode, capacity=None if capacity < 0 else capacity,
                                  feat=feat, opacity=opacity)
        d_xy, _d_conic, d_feat, d_opacity, d_scale, d_rot = _raster.render_backward(
            b, _raster.aligned(feat, 4), opacity, scale, rot, grad.contiguous().float())
    if d_opacity is None:
        d_opacity = xy.new_zeros((0,))
    return d_xy, d_scale, d_rot, d_feat, d_opacity


@rasterize_sum_backward.register_fake
def _rasterize_sum_backward_fake(xy, scale, rot, feat, opacity, grad, h, w, mode, capacity):
    d_op = xy.new_empty((xy.shape[0],)) if opacity is not None else xy.new_empty((0,))
    return (xy.new_empty(xy.shape), scale.new_empty(scale.shape), rot.new_empty(rot.shape),
            feat.new_empty(feat.shape), d_op)


def _setup_context(ctx, inputs, output):
    xy, scale, rot, feat, opacity, h, w, mode, capacity = inputs
    ctx.save_for_backward(xy, scale, rot, feat, opacity)
    ctx.meta = (h, w, mode, capacity)


def _backward(ctx, grad):
    xy, scale, rot, feat, opacity = ctx.saved_tensors
    h, w, mode, capacity = ctx.meta
    d_xy, d_scale, d_rot, d_feat, d_opacity = rasterize_sum_backward(xy, scale, rot, feat, opacity, grad, h, w,
                                                                     mode, capacity)
    return d_xy, d_scale, d_rot, d_feat, (d_opacity if opacity is not None else None), None, None, None, None


rasterize_sum.register_autograd(_backward, setup_context=_setup_context)
