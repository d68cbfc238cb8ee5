"""OSS custom rasterizer -- autograd Function over the B200 C-ABI kernels.

Drop-in for reference oss/cuda/oss_cuda/rasterizer.py: the same
``rasterize_gaussians(xy, scale, rot, feat, h, w, tile_size=16, topk_norm=True)``
call and ``_COMPILED`` / ``_C`` attributes.  The backward is the deterministic
per-pair reduction (no atomics) over the forward's own binning, fused with
the d_conic -> (d_scale, d_rot) chain rule.

Keyword-only additions (defaults keep the reference call's results):
  binning     "exact" (default) | "tight3sigma" | "full"
  opacity     (N,) tensor folded into feat as feat * opacity[:, None], with its
              gradient returned (the fold gaussian_temporal/rasterizer.py:47 does
              in PyTorch)
  blend       "sum" (default, the reference's additive weighted sum) | "alpha"
              (front-to-back compositing, a mode the reference does not have:
              a = min(0.99, opacity exp(-q/2)), skip a < 1/255, stop before the
              transmittance would fall below 1e-4, out = C + T background)
  depth       (N,) tensor ordering each tile's list front to back (alpha only;
              None keeps gid order)
  background  scalar or F values composited behind (alpha only; default 0)
  pair_capacity
              opt-in launch without any host synchronisation: the tile lists are
              sized for this many (Gaussian, tile) pairs and the device checks the
              real total; above it the lists are emptied (zero image and
              gradients) and a sticky flag is raised, read with
              oss_cuda.pair_capacity_overflowed() (e.g. together with the loss)
"""
from __future__ import annotations

from importlib import import_module

import torch
from torch.autograd import Function

from . import _raster

try:
    from . import _C

    _COMPILED = True
except ImportError:
    try:
        _C = import_module("oss_cuda._C")
        _COMPILED = True
    except ImportError:
        _C = None
        _COMPILED = False


class _RasterizeGaussians(Function):
    @staticmethod
    def forward(ctx, xy, scale, rot, feat, opacity, h, w, tile_size, topk_norm, mode, capacity):
        if not _COMPILED:
            raise RuntimeError(
                "oss_cuda extension not compiled. Run: python open-supersampling_b200/build.py"
            )
        del topk_norm
        with torch.cuda.device(xy.device):
            b = _raster.bin_gaussians(xy, scale, rot, h, w, mode, capacity=capacity, feat=feat, opacity=opacity)
            # the entry records the backward reads are written only when a gradient can follow
            if any(ctx.needs_input_grad[:5]):
                out, records, slots = _raster.render_forward(b, _raster.aligned(feat, 4), opacity, records=True)
            else:
                out, records, slots = _raster.render_forward(b, _raster.aligned(feat, 4), opacity), None, None
        ctx.save_for_backward(xy, scale, rot, feat, opacity, b.conic, b.aabb, b.pair_offset, b.geo, b.gid_sorted,
                              b.tile_offsets, records, slots)
        ctx.meta = (b.n, b.h, b.w, b.mode, b.total_pairs)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (xy, scale, rot, feat, opacity, conic, aabb, pair_offset, geo, gid_sorted, tile_offsets, records,
         slots) = ctx.saved_tensors
        n, h, w, mode, total_pairs = ctx.meta
        b = _raster.Binned(n, h, w, mode, conic, aabb, pair_offset, geo, total_pairs, gid_sorted, tile_offsets)
        grad = grad_out.contiguous()
        if grad.dtype != torch.float32:
            grad = grad.float()
        with torch.cuda.device(xy.device):
            d_xy, _d_conic, d_feat, d_opacity, d_scale, d_rot = _raster.render_backward(
                b, _raster.aligned(feat, 4), opacity, scale, rot, grad, records, slots
            )
        return d_xy, d_scale, d_rot, d_feat, d_opacity, None, None, None, None, None, None


class _RasterizeGaussiansAlpha(Function):
    @staticmethod
    def forward(ctx, xy, scale, rot, feat, opacity, depth, background, h, w, mode, capacity):
        if not _COMPILED:
            raise RuntimeError(
                "oss_cuda extension not compiled. Run: python open-supersampling_b200/build.py"
            )
        with torch.cuda.device(xy.device):
            b = _raster.bin_gaussians(xy, scale, rot, h, w, mode, depth=depth, capacity=capacity)
            bg = _raster.background_vector(background, int(feat.size(1)), xy.device)
            out, t_final, n_contrib = _raster.render_alpha_forward(b, _raster.aligned(feat, 4), opacity, bg)
        ctx.save_for_backward(xy, scale, rot, feat, opacity, bg, b.conic, b.aabb, b.pair_offset, b.geo, b.gid_sorted,
                              b.tile_offsets, t_final, n_contrib)
        ctx.meta = (b.n, b.h, b.w, b.mode, b.total_pairs)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (xy, scale, rot, feat, opacity, bg, conic, aabb, pair_offset, geo, gid_sorted, tile_offsets, t_final,
         n_contrib) = ctx.saved_tensors
        n, h, w, mode, total_pairs = ctx.meta
        b = _raster.Binned(n, h, w, mode, conic, aabb, pair_offset, geo, total_pairs, gid_sorted, tile_offsets)
        grad = grad_out.contiguous()
        if grad.dtype != torch.float32:
            grad = grad.float()
        with torch.cuda.device(xy.device):
            d_xy, _d_conic, d_feat, d_opacity, d_scale, d_rot = _raster.render_alpha_backward(
                b, _raster.aligned(feat, 4), opacity, bg, scale, rot, t_final, n_contrib, grad
            )
        return (d_xy, d_scale, d_rot, d_feat, d_opacity if opacity is not None else None, None, None, None, None,
                None, None)


def rasterize_gaussians(xy, scale, rot, feat, h, w, tile_size=16, topk_norm=True, *, binning=None, opacity=None,
                        blend="sum", depth=None, background=None, pair_capacity=None):
    """Render (F, H, W) on the GPU, differentiably: sum_g feat[g] * exp(-q_g / 2)
    (blend="sum", the reference op) or front-to-back compositing (blend="alpha").

    Reference: oss/cuda/oss_cuda/rasterizer.py:68-70.
    """
    h, w, tile_size = int(h), int(w), int(tile_size)
    _raster.check_gaussians(xy, scale, rot, feat)
    _raster.check_hw(h, w, tile_size)
    if opacity is not None:
        _raster.check_float_cuda(opacity, "opacity")
        if opacity.dim() != 1 or opacity.size(0) != xy.size(0):
            raise RuntimeError("opacity must be (N,)")
    mode = _raster.binning_mode(binning)
    if pair_capacity is not None:
        pair_capacity = int(pair_capacity)
        if pair_capacity < 0 or pair_capacity > _raster.INT32_MAX:
            raise ValueError("pair_capacity must be in [0, 2**31 - 1]")
    if blend == "sum":
        if depth is not None or background is not None:
            raise ValueError("depth and background apply to blend='alpha' only")
        return _RasterizeGaussians.apply(xy, scale, rot, feat, opacity, h, w, tile_size, bool(topk_norm), mode,
                                         pair_capacity)
    if blend != "alpha":
        raise ValueError(f"blend must be 'sum' or 'alpha', got {blend!r}")
    if depth is not None:
        _raster.check_float_cuda(depth, "depth")
        if depth.dim() != 1 or depth.size(0) != xy.size(0):
            raise RuntimeError("depth must be (N,)")
    return _RasterizeGaussiansAlpha.apply(xy, scale, rot, feat, opacity, depth, background, h, w, mode,
                                          pair_capacity)
