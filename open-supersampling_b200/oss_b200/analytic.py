"""Analytic-Splatting pixel integral on the B200 kernels.

Drop-in for oss/sr/v6/aa_analytic_splat.py (``analytic_pixel_integral``,
``logistic_cdf``): the same signatures, broadcasting, output dtype and error
messages, computed elementwise in liboss_b200.so (csrc/analytic.cu) in fp32,
with a backward that is the chain rule of the closed-form 2x2 eigensystem, the
rotation and the per-axis logistic-CDF integrals (the isotropic branch below
an eigengap of 1e-5 included).
"""
from __future__ import annotations

import torch

from oss_cuda import _lib
from oss_cuda._raster import stream_of

__all__ = ["analytic_pixel_integral", "logistic_cdf"]


def _need_cuda(t: torch.Tensor) -> None:
    if t.device.type != "cuda":
        raise RuntimeError("the analytic pixel integral runs on liboss_b200.so and needs CUDA tensors")


class _Logistic(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        xf = x.detach().to(torch.float32).contiguous()
        out = torch.empty_like(xf)
        _lib.check(_lib.lib().oss_logistic_cdf(xf.numel(), xf.data_ptr(), None, out.data_ptr(), stream_of(xf)),
                   "oss_logistic_cdf")
        ctx.save_for_backward(xf)
        ctx.dtype = x.dtype
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        (xf,) = ctx.saved_tensors
        gf = g.detach().to(torch.float32).contiguous()
        out = torch.empty_like(xf)
        _lib.check(_lib.lib().oss_logistic_cdf(xf.numel(), xf.data_ptr(), gf.data_ptr(), out.data_ptr(),
                                               stream_of(xf)), "oss_logistic_cdf")
        return out.to(ctx.dtype)


def logistic_cdf(x: torch.Tensor) -> torch.Tensor:
    """S(x) = 1 / (1 + exp(-1.6 x - 0.07 x^3)) (aa_analytic_splat.py:46-57)."""
    _need_cuda(x)
    return _Logistic.apply(x)


class _Integral(torch.autograd.Function):
    @staticmethod
    def forward(ctx, dx, dy, s00, s01, s10, s11):
        ins = [t.detach().to(torch.float32).contiguous() for t in (dx, dy, s00, s01, s10, s11)]
        out = torch.empty_like(ins[0])
        _lib.check(_lib.lib().oss_analytic_pixel_integral(out.numel(), *(t.data_ptr() for t in ins), out.data_ptr(),
                                                          stream_of(out)), "oss_analytic_pixel_integral")
        ctx.save_for_backward(*ins)
        ctx.dtypes = tuple(t.dtype for t in (dx, dy, s00, s01, s10, s11))
        return out

    @staticmethod
    def backward(ctx, g):
        ins = ctx.saved_tensors
        gf = g.detach().to(torch.float32).contiguous()
        grads = [torch.empty_like(ins[0]) for _ in range(6)]
        _lib.check(_lib.lib().oss_analytic_pixel_integral_backward(gf.numel(), *(t.data_ptr() for t in ins),
                                                                   gf.data_ptr(), *(t.data_ptr() for t in grads),
                                                                   stream_of(gf)),
                   "oss_analytic_pixel_integral_backward")
        return tuple(t.to(d) for t, d in zip(grads, ctx.dtypes))


def analytic_pixel_integral(delta_x: torch.Tensor, delta_y: torch.Tensor, sigma_2d_inv: torch.Tensor) -> torch.Tensor:
    """Pixel-area integral of an un-normalised 2D Gaussian (aa_analytic_splat.py:72-202):
    offsets (..., P) broadcast against per-Gaussian inverse covariances (..., 2, 2)
    (trailing pixel axes appended to the matrices' batch shape); returns the
    broadcast shape in sigma_2d_inv's dtype."""
    if sigma_2d_inv.shape[-2:] != (2, 2):
        raise ValueError(f"sigma_2d_inv must be (..., 2, 2), got {tuple(sigma_2d_inv.shape)}")
    _need_cuda(sigma_2d_inv)
    in_dtype = sigma_2d_inv.dtype
    dx, dy = torch.broadcast_tensors(delta_x, delta_y)
    entries = [sigma_2d_inv[..., 0, 0], sigma_2d_inv[..., 0, 1], sigma_2d_inv[..., 1, 0], sigma_2d_inv[..., 1, 1]]
    aligned = []
    for e in entries:
        while e.ndim < dx.ndim:
            e = e.unsqueeze(-1)
        aligned.append(e)
    parts = torch.broadcast_tensors(dx, dy, *aligned)
    return _Integral.apply(*parts).to(in_dtype)
