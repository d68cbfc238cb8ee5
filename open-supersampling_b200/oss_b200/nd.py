"""v7 N-D Gaussian time-slice rasterizer on the B200 kernels.

Drop-in for oss/sr/v7/nd_rasterizer.py (``render_nd_time_slice``,
``time_marginal``, ``NDGaussian``): the same signatures and math.  Per
Gaussian, on the device with PyTorch ops (differentiable):
  * Mip-Splatting 3D smoothing: cov + v3 I, opacity * sqrt(det cov / det(cov + v3 I));
  * conditioning on t = t_query: mean_xy + cov_xt (t_query - mean_t) / cov_tt, the
    Schur complement cov_xy - cov_xt cov_xt^T / cov_tt and the marginal density
    of t_query (cov_tt clamped at 1e-12);
  * Mip 2D filter: cov_2d + v2 I, weight * sqrt(det cov_2d / det(cov_2d + v2 I)).
The splat -- the part that touches every pixel -- runs in liboss_b200.so
(csrc/nd.cu) through tile lists: each Gaussian adds feat * opacity * weight *
exp(-q/2) at pixel centres (j + 0.5, i + 0.5) inside its cull box of 3 sqrt(largest
eigenvalue) around the conditioned mean, as the reference's loop bounds
(nd_rasterizer.py:107-165).  Its backward comes from the per-pair kernel and the
per-Gaussian reduce of the additive path; PyTorch's autograd carries the
gradients back through the per-Gaussian steps above.
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


def _det3(c: torch.Tensor) -> torch.Tensor:
    return (c[..., 0, 0] * (c[..., 1, 1] * c[..., 2, 2] - c[..., 1, 2] * c[..., 2, 1])
            - c[..., 0, 1] * (c[..., 1, 0] * c[..., 2, 2] - c[..., 1, 2] * c[..., 2, 0])
            + c[..., 0, 2] * (c[..., 1, 0] * c[..., 2, 1] - c[..., 1, 1] * c[..., 2, 0]))


def _det2(c: torch.Tensor) -> torch.Tensor:
    return c[..., 0, 0] * c[..., 1, 1] - c[..., 0, 1] * c[..., 1, 0]


def _smooth3(covs: torch.Tensor, opacities: torch.Tensor, variance: float):
    """Mip-Splatting 3D smoothing (nd_rasterizer.py:168-209), in fp32."""
    if variance <= 0:
        return covs, opacities
    c = covs.float()
    s = c + variance * torch.eye(3, device=c.device, dtype=torch.float32)
    factor = torch.sqrt(_det3(c).clamp(min=1e-12) / _det3(s).clamp(min=1e-12))
    return s.to(covs.dtype), opacities * factor.to(opacities.dtype)


def _mip2(cov2: torch.Tensor, weights: torch.Tensor, variance: float):
    """Mip-Splatting 2D filter (nd_rasterizer.py:212-239), in fp32."""
    if variance <= 0:
        return cov2, weights
    c = cov2.float()
    s = c + variance * torch.eye(2, device=c.device, dtype=torch.float32)
    factor = torch.sqrt(_det2(c).clamp(min=1e-12) / _det2(s).clamp(min=1e-12))
    return s.to(cov2.dtype), weights * factor.to(weights.dtype)


def _cull_boxes(mean_xy: torch.Tensor, cov2: torch.Tensor, h: int, w: int) -> torch.Tensor:
    """(N, 4) int32 boxes [x0, x1) x [y0, y1) of 3 sqrt(largest eigenvalue, at least
    1e-6) around the mean, clipped to the frame (nd_rasterizer.py:117-124); the
    bounds come from the fp32 eigenvalue and fp64 floor / ceil, as the
    reference's Python arithmetic on .item() values."""
    with torch.no_grad():
        c = cov2.float()
        a, b, d = c[:, 0, 0], 0.5 * (c[:, 0, 1] + c[:, 1, 0]), c[:, 1, 1]
        half = 0.5 * (a - d)
        lam = (0.5 * (a + d) + torch.sqrt(half * half + b * b)).clamp(min=1e-6)
        r = 3.0 * torch.sqrt(lam).double()
        m = mean_xy.detach().double()
        x0 = torch.floor(m[:, 0] - r).clamp(min=0)
        x1 = torch.minimum(torch.ceil(m[:, 0] + r), torch.full_like(r, float(w)))
        y0 = torch.floor(m[:, 1] - r).clamp(min=0)
        y1 = torch.minimum(torch.ceil(m[:, 1] + r), torch.full_like(r, float(h)))
        box = torch.stack([x0, y0, x1, y1], dim=-1)
        box = torch.nan_to_num(box, nan=0.0, posinf=0.0, neginf=0.0).clamp(-2**30, 2**30)
        return box.to(torch.int32).contiguous()


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
    covs_f, op_f = _smooth3(covs, opacities, mip_3d_variance)
    mean_c, cov_c, weight_t = time_marginal(means, covs_f, t_query)
    weights = weight_t if time_falloff else torch.ones_like(weight_t)
    cov_c, weights = _mip2(cov_c, weights, mip_2d_variance)
    n = means.shape[0]
    r = features.shape[1]
    if n == 0 or r == 0:
        return torch.zeros((r, h, w), device=means.device, dtype=dtype)
    c = cov_c.float()
    det = c[:, 0, 0] * c[:, 1, 1] - c[:, 0, 1] * c[:, 1, 0]
    conic = torch.stack([c[:, 1, 1] / det, -c[:, 0, 1] / det, c[:, 0, 0] / det], dim=-1)
    amp = (op_f.float() * weights.float())
    box = _cull_boxes(mean_c, c, h, w)
    xy = mean_c.float()
    feat = features.float()
    parts = [_NDSplat.apply(xy, conic, amp, feat[:, k:k + _MAX_F], box, h, w) for k in range(0, r, _MAX_F)]
    return (parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)).to(dtype)
