"""v7 N-D Gaussian time-slice rasterizer on the B200 kernels.

Drop-in for oss/sr/v7/nd_rasterizer.py (``render_nd_time_slice``,
``time_marginal``, ``NDGaussian``): the same signatures and math, in two
autograd steps that both run in liboss_b200.so (csrc/nd.cu):
  * per Gaussian, one kernel: Mip-Splatting 3D smoothing (cov + v3 I, opacity *
    sqrt(det cov / det(cov + v3 I))), conditioning on t = t_query (mean_xy +
    cov_xt (t_query - mean_t) / cov_tt, the Schur complement cov_xy - cov_xt
    cov_xt^T / cov_tt and the marginal density of t_query, cov_tt clamped at
    1e-12), the Mip 2D filter (cov_2d + v2 I, weight * sqrt(det cov_2d /
    det(cov_2d + v2 I))), the inverse covariance and the cull box of 3 sqrt(largest
    eigenvalue) around the conditioned mean (nd_rasterizer.py:117-124); its
    backward is the chain rule of these steps written out;
  * the splat through tile lists: each Gaussian adds feat * opacity * weight *
    exp(-q/2) at pixel centres (j + 0.5, i + 0.5) inside its cull box
    (nd_rasterizer.py:107-165); its backward is the per-pair kernel and the
    per-Gaussian reduce of the additive path.
``time_marginal`` is also given as PyTorch ops for callers that use it alone.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Tuple

import torch

from oss_cuda import _lib
from oss_cuda._raster import aligned, check_hw, read_total, stream_of

__all__ = ["NDGaussian", "render_nd_time_slice", "time_marginal"]

_MAX_F = 32  # channels per splat launch; wider features run in chunks


@dataclass
class NDGaussian:
    """One 3D (x, y, t) Gaussian (nd_rasterizer.py:40-50)."""

    mean: torch.Tensor
    cov: torch.Tensor
    feature: torch.Tensor
    opacity: torch.Tensor


def time_marginal(mean: torch.Tensor, cov: torch.Tensor, t_query: float):
    """(mean_xy | t, cov_xy | t, density of t_query) for (..., 3) means and
    (..., 3, 3) covariances (nd_rasterizer.py:53-104)."""
    vtt = cov[..., 2, 2].clamp(min=1e-12)
    vxt = cov[..., :2, 2]
    dt = float(t_query) - mean[..., 2]
    mean_c = mean[..., :2] + vxt * (dt / vtt).unsqueeze(-1)
    cov_c = cov[..., :2, :2] - (vxt.unsqueeze(-1) * vxt.unsqueeze(-2)) / vtt[..., None, None]
    log_w = -0.5 * dt * dt / vtt - 0.5 * (math.log(2.0 * math.pi) + vtt.log())
    return mean_c, cov_c, log_w.exp()


class _NDCondition(torch.autograd.Function):
    """(means, covs, opacities) -> (xy, conic, amp, box) in one kernel per
    direction (csrc/nd.cu): the Mip 3D filter, the conditioning on t_query and
    the Mip 2D filter of the functions above, with their chain rule by hand."""

    @staticmethod
    def forward(ctx, means, covs, opac, t_query, falloff, v3, v2, h, w):
        lib = _lib.lib()
        n = int(means.shape[0])
        dev = means.device
        m = means.detach().to(torch.float32).contiguous()
        c = covs.detach().to(torch.float32).reshape(n, 9).contiguous()
        o = opac.detach().to(torch.float32).contiguous()
        xy = torch.empty((n, 2), device=dev, dtype=torch.float32)
        conic = torch.empty((n, 3), device=dev, dtype=torch.float32)
        amp = torch.empty((n,), device=dev, dtype=torch.float32)
        box = torch.empty((n, 4), device=dev, dtype=torch.int32)
        _lib.check(lib.oss_nd_condition(n, h, w, m.data_ptr(), c.data_ptr(), o.data_ptr(), float(t_query),
                                        int(bool(falloff)), float(v3), float(v2), xy.data_ptr(), conic.data_ptr(),
                                        amp.data_ptr(), box.data_ptr(), stream_of(m)), "oss_nd_condition")
        ctx.save_for_backward(m, c, o)
        ctx.params = (float(t_query), int(bool(falloff)), float(v3), float(v2))
        ctx.dtypes = (means.dtype, covs.dtype, opac.dtype)
        ctx.mark_non_differentiable(box)
        return xy, conic, amp, box

    @staticmethod
    def backward(ctx, g_xy, g_conic, g_amp, _g_box):
        lib = _lib.lib()
        m, c, o = ctx.saved_tensors
        n = int(m.shape[0])
        tq, falloff, v3, v2 = ctx.params
        z = lambda g, shape: (g if g is not None else torch.zeros(shape, device=m.device)).to(torch.float32).contiguous()
        gx, gc, ga = z(g_xy, (n, 2)), z(g_conic, (n, 3)), z(g_amp, (n,))
        d_m = torch.empty_like(m)
        d_c = torch.empty_like(c)
        d_o = torch.empty_like(o)
        _lib.check(lib.oss_nd_condition_backward(n, m.data_ptr(), c.data_ptr(), o.data_ptr(), tq, falloff, v3, v2,
                                                 gx.data_ptr(), gc.data_ptr(), ga.data_ptr(), d_m.data_ptr(),
                                                 d_c.data_ptr(), d_o.data_ptr(), stream_of(m)),
                   "oss_nd_condition_backward")
        dm, dc, do = ctx.dtypes
        return d_m.to(dm), d_c.reshape(n, 3, 3).to(dc), d_o.to(do), None, None, None, None, None, None


class _NDSplat(torch.autograd.Function):
    """(xy, conic (a, b, d), amplitude, features) of 2D Gaussians with cull boxes ->
    (F, H, W), through csrc/nd.cu; F <= 32."""

    @staticmethod
    def forward(ctx, xy, conic, amp, feat, box, h, w):
        lib = _lib.lib()
        n, f = int(xy.shape[0]), int(feat.shape[1])
        dev = xy.device
        _, _, tiles, _ = check_hw(h, w, _lib.TILE)
        xy, conic, amp = aligned(xy.contiguous(), 8), conic.contiguous(), amp.contiguous()
        feat, box = feat.contiguous(), aligned(box, 16)
        f32, i32 = dict(device=dev, dtype=torch.float32), dict(device=dev, dtype=torch.int32)
        aabb = torch.empty((n, 4), **i32)
        pair_offset = torch.empty((n + 1,), **i32)
        geo = torch.empty((n, 8), **f32)
        prec = torch.empty((max(1, n), lib.oss_nd_record_floats(f)), **f32)
        total = torch.empty((1,), device=dev, dtype=torch.int64)
        tile_count = torch.empty((max(1, lib.oss_tile_count_elems(tiles)),), **i32)
        tile_offsets = torch.empty((tiles + 1,), **i32)
        scratch = torch.empty((max(1, lib.oss_render_prepare_scratch_bytes(n)),), device=dev, dtype=torch.uint8)
        s = stream_of(xy)
        _lib.check(lib.oss_nd_prepare(n, h, w, xy.data_ptr(), conic.data_ptr(), box.data_ptr(), f, feat.data_ptr(),
                                      amp.data_ptr(), aabb.data_ptr(), pair_offset.data_ptr(), geo.data_ptr(),
                                      prec.data_ptr(), total.data_ptr(), tile_count.data_ptr(), tile_offsets.data_ptr(),
                                      scratch.data_ptr(), scratch.numel(), s), "oss_nd_prepare")
        pairs = read_total(total, s)
        gid = torch.empty((max(1, pairs),), **i32)
        overflow = torch.empty((1,), **i32)
        scratch2 = torch.empty((max(1, lib.oss_bin_pairs_scratch_bytes(n, pairs, tiles)),), device=dev,
                               dtype=torch.uint8)
        _lib.check(lib.oss_bin_pairs(n, h, w, _lib.OSS_BIN_TIGHT3SIGMA, aabb.data_ptr(), pair_offset.data_ptr(),
                                     tile_count.data_ptr(), total.data_ptr(), pairs, None, None, gid.data_ptr(),
                                     tile_offsets.data_ptr(), overflow.data_ptr(), scratch2.data_ptr(),
                                     scratch2.numel(), s), "oss_bin_pairs")
        image = torch.empty((f, h, w), **f32)
        _lib.check(lib.oss_nd_forward(f, h, w, prec.data_ptr(), box.data_ptr(), gid.data_ptr(),
                                      tile_offsets.data_ptr(), image.data_ptr(), s), "oss_nd_forward")
        ctx.save_for_backward(prec, box, gid, tile_offsets, aabb, pair_offset, geo, feat, amp)
        ctx.dims = (n, f, h, w, pairs)
        return image

    @staticmethod
    def backward(ctx, grad_image):
        lib = _lib.lib()
        prec, box, gid, tile_offsets, aabb, pair_offset, geo, feat, amp = ctx.saved_tensors
        n, f, h, w, pairs = ctx.dims
        dev = geo.device
        go = grad_image.detach().to(torch.float32).contiguous()
        stride = lib.oss_pair_grad_stride(f)
        pairgrad = torch.zeros((max(1, pairs), stride), device=dev, dtype=torch.float32)
        s = stream_of(geo)
        _lib.check(lib.oss_nd_backward_pairs(f, h, w, prec.data_ptr(), box.data_ptr(), gid.data_ptr(),
                                             tile_offsets.data_ptr(), aabb.data_ptr(), pair_offset.data_ptr(),
                                             go.data_ptr(), pairgrad.data_ptr(), s), "oss_nd_backward_pairs")
        d_xy = torch.empty((n, 2), device=dev, dtype=torch.float32)
        d_conic = torch.empty((n, 3), device=dev, dtype=torch.float32)
        d_feat = torch.empty((n, f), device=dev, dtype=torch.float32)
        d_amp = torch.empty((n,), device=dev, dtype=torch.float32)
        _lib.check(lib.oss_reduce_pair_grads(n, f, pairgrad.data_ptr(), pair_offset.data_ptr(), geo.data_ptr(),
                                             feat.data_ptr(), amp.data_ptr(), None, None, d_xy.data_ptr(),
                                             d_conic.data_ptr(), d_feat.data_ptr(), d_amp.data_ptr(), None, None, s),
                   "oss_reduce_pair_grads")
        return d_xy, d_conic, d_amp, d_feat, None, None, None


def render_nd_time_slice(means: torch.Tensor, covs: torch.Tensor, features: torch.Tensor, opacities: torch.Tensor,
                         t_query: float, image_hw: Tuple[int, int], time_falloff: bool = True,
                         mip_3d_variance: float = 0.2, mip_2d_variance: float = 0.1) -> torch.Tensor:
    """(R, H, W) feature image of the N-D mixture at time t_query
    (nd_rasterizer.py:242-281).  Differentiable in means, covs, features and
    opacities; CUDA tensors."""
    if means.ndim != 2 or means.shape[1] != 3:
        raise ValueError(f"means must be (N, 3); got {tuple(means.shape)}")
    if covs.shape != (means.shape[0], 3, 3):
        raise ValueError(f"covs must be (N, 3, 3); got {tuple(covs.shape)}")
    if features.ndim != 2 or features.shape[0] != means.shape[0]:
        raise ValueError(f"features must be (N, R); got {tuple(features.shape)}")
    if means.device.type != "cuda":
        raise RuntimeError("render_nd_time_slice runs on liboss_b200.so and needs CUDA tensors")
    h, w = int(image_hw[0]), int(image_hw[1])
    dtype = features.dtype
    n = means.shape[0]
    r = features.shape[1]
    if n == 0 or r == 0:
        return torch.zeros((r, h, w), device=means.device, dtype=dtype)
    xy, conic, amp, box = _NDCondition.apply(means, covs, opacities, float(t_query), bool(time_falloff),
                                             float(mip_3d_variance), float(mip_2d_variance), h, w)
    feat = features.float()
    parts = [_NDSplat.apply(xy, conic, amp, feat[:, k:k + _MAX_F], box, h, w) for k in range(0, r, _MAX_F)]
    return (parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)).to(dtype)
