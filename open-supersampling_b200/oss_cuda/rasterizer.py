"""OSS custom rasterizer -- autograd Function over the B200 C-ABI kernels.

Drop-in for reference oss/cuda/oss_cuda/rasterizer.py: the same
``rasterize_gaussians(xy, scale, rot, feat, h, w, tile_size=16, topk_norm=True)``
call and ``_COMPILED`` / ``_C`` attributes.  The backward is the deterministic
per-pair reduction (no atomics) over the forward's own binning, fused with
the d_conic -> (d_scale, d_rot) chain rule.

Keyword-only additions (defaults keep the reference call's results):
  binning     "exact56" (default: q <= 56 lists, weights left out < 6.9e-13) |
              "exact" (q <= 176: every nonzero fp32 weight) | "tight3sigma" | "full"
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
  weight      "gaussian" (default, exp(-q/2)) | "analytic" (the Analytic-Splatting
              pixel integral of oss/sr/v6/aa_analytic_splat.py, blend="sum")
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

from . import _batched, _feather, _lib, _raster, ops

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


class _RasterizeGaussiansAnalytic(Function):
    """The additive render with the Analytic-Splatting pixel integral as weight."""

    @staticmethod
    def forward(ctx, xy, scale, rot, feat, opacity, h, w, mode):
        if not _COMPILED:
            raise RuntimeError(
                "oss_cuda extension not compiled. Run: python open-supersampling_b200/build.py"
            )
        with torch.cuda.device(xy.device):
            b = _raster.bin_gaussians(xy, scale, rot, h, w, mode)
            out = _raster.render_analytic_forward(b, _raster.aligned(feat, 4), opacity)
        ctx.save_for_backward(xy, scale, rot, feat, opacity, b.conic, b.aabb, b.pair_offset, b.geo, b.gid_sorted,
                              b.tile_offsets)
        ctx.meta = (b.n, b.h, b.w, b.mode, b.total_pairs)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        xy, scale, rot, feat, opacity, conic, aabb, pair_offset, geo, gid_sorted, tile_offsets = ctx.saved_tensors
        n, h, w, mode, total_pairs = ctx.meta
        b = _raster.Binned(n, h, w, mode, conic, aabb, pair_offset, geo, total_pairs, gid_sorted, tile_offsets)
        grad = grad_out.contiguous().float()
        with torch.cuda.device(xy.device):
            d_xy, _d_conic, d_feat, d_opacity, d_scale, d_rot = _raster.render_analytic_backward(
                b, _raster.aligned(feat, 4), opacity, scale, rot, grad)
        return d_xy, d_scale, d_rot, d_feat, d_opacity, None, None, None


def rasterize_gaussians(xy, scale, rot, feat, h, w, tile_size=16, topk_norm=True, *, binning=None, opacity=None,
                        blend="sum", depth=None, background=None, pair_capacity=None, overlap=0,
                        phase_offset=(0, 0), weight="gaussian"):
    """Render (F, H, W) on the GPU, differentiably: sum_g feat[g] * exp(-q_g / 2)
    (blend="sum", the reference op) or front-to-back compositing (blend="alpha").

    Reference: oss/cuda/oss_cuda/rasterizer.py:68-70.  The keywords add the
    build's options; left at their defaults they do not change the result:
    binning (tile lists), opacity (folded in the kernel), blend / depth /
    background (alpha compositing), pair_capacity (no host sync), overlap (the
    4-phase feathered overlapping-tile render of oss/sr/v6/rasterizer.py:159-242,
    blend="sum"), phase_offset = (dx, dy) integer pixels added to every mean
    before rendering (the per-frame spawner offset, oss/sr/v6/model.py:795-820)
    and weight="analytic", the Analytic-Splatting pixel integral of
    oss/sr/v6/aa_analytic_splat.py in place of exp(-q/2) (blend="sum", F <= 32).
    """
    h, w, tile_size = int(h), int(w), int(tile_size)
    dx, dy = (int(v) for v in phase_offset)
    if dx or dy:
        xy = xy + torch.tensor([float(dx), float(dy)], device=xy.device, dtype=xy.dtype)
    overlap = int(overlap)
    if overlap < 0:
        raise ValueError(f"overlap must be >= 0; got {overlap}")
    if overlap > 0:
        if blend != "sum":
            raise ValueError("overlap applies to blend='sum' only")
        _raster.check_gaussians(xy, scale, rot, feat)
        _raster.check_hw(h, w, tile_size)
        if weight == "gaussian" and _feather.supported(overlap, int(feat.size(1)), h, w):
            # one pass: every Gaussian once, with its separable feather window
            if opacity is not None:
                _raster.check_float_cuda(opacity, "opacity")
                if opacity.dim() != 1 or opacity.size(0) != xy.size(0):
                    raise RuntimeError("opacity must be (N,)")
            if pair_capacity is not None:
                pair_capacity = int(pair_capacity)
                if pair_capacity < 0 or pair_capacity > _raster.INT32_MAX:
                    raise ValueError("pair_capacity must be in [0, 2**31 - 1]")
            return _feather.RasterizeFeathered.apply(xy, scale, rot, feat, opacity, h, w, _raster.binning_mode(binning),
                                                     overlap, pair_capacity)
        # wider channel counts or overlaps: the reference's composition of four phase renders
        from .overlap import render_overlapped_with

        def one(x, s, r, f, hh, ww):
            return rasterize_gaussians(x, s, r, f, hh, ww, tile_size, topk_norm, binning=binning, opacity=opacity,
                                       pair_capacity=pair_capacity, weight=weight)

        return render_overlapped_with(one, xy, scale, rot, feat, h, w, overlap)
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
    if weight not in ("gaussian", "analytic"):
        raise ValueError(f"weight must be 'gaussian' or 'analytic', got {weight!r}")
    if weight == "analytic":
        if blend != "sum" or pair_capacity is not None:
            raise ValueError("weight='analytic' applies to blend='sum' without pair_capacity")
        if int(feat.size(1)) > 32:
            raise ValueError("weight='analytic' renders at most 32 channels per call")
        # the logistic tails of the analytic weight outlast exp(-q/2): its default lists are q <= 176
        mode = _raster.binning_mode(binning, default="exact")
        return _RasterizeGaussiansAnalytic.apply(xy, scale, rot, feat, opacity, h, w, mode)
    if blend == "sum":
        if depth is not None or background is not None:
            raise ValueError("depth and background apply to blend='alpha' only")
        if torch.compiler.is_compiling():
            # traced by torch.compile: the dispatcher-visible operator (oss_cuda.ops)
            return ops.rasterize_sum(xy, scale, rot, feat, opacity, h, w, mode,
                                     -1 if pair_capacity is None else pair_capacity)
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


def rasterize_gaussians_batched(xy, scale, rot, feat, offsets, h, w, tile_size=16, topk_norm=True, **kwargs):
    """B frames in one call, frame b drawn from Gaussians [offsets[b], offsets[b+1])
    of the concatenated inputs: (B, F, H, W), differentiable like
    rasterize_gaussians (keywords as there; opacity and depth are per Gaussian of
    the concatenation).  offsets is a host sequence or CPU tensor of B+1
    non-decreasing ints from 0 to N.

    The additive render (blend="sum", the Gaussian weight, culled lists, no
    overlap or phase offset) runs as one launch chain over all B frames
    (oss_cuda._batched), with the same images and gradients as B calls; the
    other modes call rasterize_gaussians once per frame."""
    offs = [int(v) for v in (offsets.tolist() if torch.is_tensor(offsets) else offsets)]
    n = int(xy.size(0))
    if len(offs) < 1 or offs[0] != 0 or offs[-1] != n or any(b < a for a, b in zip(offs, offs[1:])):
        raise ValueError("offsets must be non-decreasing from 0 to N")
    h, w, tile_size = int(h), int(w), int(tile_size)
    if len(offs) > 1 and _one_chain(kwargs):
        _raster.check_gaussians(xy, scale, rot, feat)
        _raster.check_hw(h, w, tile_size)
        opacity = kwargs.get("opacity")
        if opacity is not None:
            _raster.check_float_cuda(opacity, "opacity")
            if opacity.dim() != 1 or opacity.size(0) != n:
                raise RuntimeError("opacity must be (N,)")
        if int(feat.size(1)) > _lib.MAX_CHANNELS:
            raise RuntimeError(f"F must be <= {_lib.MAX_CHANNELS}")
        mode = _raster.binning_mode(kwargs.get("binning"))
        capacity = kwargs.get("pair_capacity")
        if capacity is not None:
            capacity = int(capacity)
            if capacity < 0 or capacity > _raster.INT32_MAX:
                raise ValueError("pair_capacity must be in [0, 2**31 - 1]")
        return _batched.RasterizeFrames.apply(xy, scale, rot, feat, opacity, tuple(offs), h, w, mode, capacity)
    per_g = {k: kwargs.pop(k) for k in ("opacity", "depth") if kwargs.get(k) is not None}
    frames = []
    for a, b in zip(offs, offs[1:]):
        kw = dict(kwargs)
        kw.update({k: v[a:b] for k, v in per_g.items()})
        frames.append(rasterize_gaussians(xy[a:b], scale[a:b], rot[a:b], feat[a:b], h, w, tile_size, topk_norm,
                                          **kw))
    if not frames:
        return torch.zeros((0, int(feat.size(1)), int(h), int(w)), device=xy.device, dtype=torch.float32)
    return torch.stack(frames, 0)


def _one_chain(kwargs) -> bool:
    """The keywords of rasterize_gaussians_batched that the one-chain path covers."""
    known = {"binning", "opacity", "pair_capacity", "blend", "weight", "overlap", "phase_offset", "depth", "background"}
    if set(kwargs) - known or torch.compiler.is_compiling():
        return False
    if kwargs.get("blend", "sum") != "sum" or kwargs.get("weight", "gaussian") != "gaussian":
        return False
    if int(kwargs.get("overlap", 0)) != 0 or tuple(int(v) for v in kwargs.get("phase_offset", (0, 0))) != (0, 0):
        return False
    if kwargs.get("depth") is not None or kwargs.get("background") is not None:
        return False
    return _raster.binning_mode(kwargs.get("binning")) != _lib.OSS_BIN_FULL
