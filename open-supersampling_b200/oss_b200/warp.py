"""Canvas warp on the GPU through liboss_b200.so.

warp_canvas   -- drop-in for oss/sr/v6/canvas_warp.py:177-254 (GS-STVSR:
                 motion sample, J = I + grad(motion), J S J^T + Sigma_recon,
                 re-decomposition, in-frame compaction), with an added
                 ``alpha`` that scales the motion (extrapolation at t + alpha).
warp_positions -- drop-in for oss/gaussian/canvas/warp.py:28-91.

warp_canvas is differentiable (its backward is a kernel of its own);
warp_positions is forward only and raises on inputs that require grad under
grad mode instead of silently cutting the graph.
"""
from __future__ import annotations

from typing import Tuple

import torch
from torch.autograd import Function

from oss_cuda import _lib
from oss_cuda._raster import aligned, stream_of

from .canvas import CanvasState


def _validate_canvas(canvas) -> int:
    # same checks and messages as canvas_warp.py:28-52
    count = int(canvas.count)
    if count < 0:
        raise ValueError(f"canvas.count must be non-negative; got {canvas.count}")
    if canvas.positions.ndim != 2 or canvas.positions.shape[-1] != 2:
        raise ValueError(f"canvas.positions must be (N, 2); got {tuple(canvas.positions.shape)}")
    if canvas.scales.ndim != 2 or canvas.scales.shape[-1] != 2:
        raise ValueError(f"canvas.scales must be (N, 2); got {tuple(canvas.scales.shape)}")
    if canvas.rotations.ndim != 1:
        raise ValueError(f"canvas.rotations must be (N,); got {tuple(canvas.rotations.shape)}")
    if canvas.opacities.ndim != 1:
        raise ValueError(f"canvas.opacities must be (N,); got {tuple(canvas.opacities.shape)}")
    if canvas.colors.ndim != 2:
        raise ValueError(f"canvas.colors must be (N, F); got {tuple(canvas.colors.shape)}")
    lengths = tuple(t.shape[0] for t in (canvas.positions, canvas.scales, canvas.rotations, canvas.opacities,
                                         canvas.colors))
    if count > min(lengths):
        raise ValueError(f"canvas.count={count} exceeds tensor lengths {lengths}")
    return count


def _validate_motion(motion_lr: torch.Tensor, output_hw) -> tuple[int, int]:
    if motion_lr.ndim != 4 or motion_lr.shape[1] != 2:
        raise ValueError(f"motion_lr must be (B, 2, H, W); got {tuple(motion_lr.shape)}")
    if motion_lr.shape[0] < 1:
        raise ValueError("motion_lr batch dimension must be non-empty")
    h_hr, w_hr = int(output_hw[0]), int(output_hw[1])
    if h_hr <= 0 or w_hr <= 0:
        raise ValueError(f"output_hw must be positive; got {output_hw}")
    return h_hr, w_hr


def _no_grad_inputs(*tensors) -> None:
    if torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors):
        raise RuntimeError("oss_b200 warp kernels are forward-only; call under torch.no_grad() or detach inputs")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return aligned(t.detach().to(dtype=torch.float32).contiguous(), 8)


def _recon4(sigma_recon) -> list[float]:
    if isinstance(sigma_recon, torch.Tensor):
        if sigma_recon.shape[-2:] != (2, 2) or sigma_recon.numel() != 4:
            raise ValueError("sigma_recon tensor must be a single (2, 2) matrix for the CUDA warp")
        return [float(v) for v in sigma_recon.detach().float().reshape(4).cpu()]
    s = float(sigma_recon)
    return [s, 0.0, 0.0, s]


class _WarpCanvas(Function):
    """The canvas warp and its backward on the GPU (oss_warp_canvas /
    oss_warp_canvas_backward): gradients reach positions, scales, rotations,
    opacities, colors and the motion field, as autograd's do through the
    reference's torch ops."""

    @staticmethod
    def forward(ctx, motion, pos, sc, rt, op, col, h, w, recon4, alpha):
        n, f = int(pos.shape[0]), int(col.shape[1])
        dev = pos.device
        lib = _lib.lib()
        f32 = dict(device=dev, dtype=torch.float32)
        outs = [torch.empty((n, 2), **f32), torch.empty((n, 2), **f32), torch.empty((n,), **f32),
                torch.empty((n,), **f32), torch.empty((n, f), **f32)]
        out_count = torch.empty((1,), device=dev, dtype=torch.int32)
        scratch = torch.empty((lib.oss_warp_canvas_scratch_bytes(n),), device=dev, dtype=torch.uint8)
        recon = torch.tensor(recon4, dtype=torch.float32)
        _lib.check(
            lib.oss_warp_canvas(n, f, motion.shape[1], motion.shape[2], h, w, motion.data_ptr(), float(alpha),
                                recon.data_ptr(), pos.data_ptr(), sc.data_ptr(), rt.data_ptr(), op.data_ptr(),
                                col.data_ptr() if f > 0 else None, *(o.data_ptr() if o.numel() else None for o in outs),
                                out_count.data_ptr(), scratch.data_ptr(), scratch.numel(), stream_of(pos)),
            "oss_warp_canvas",
        )
        k = int(out_count.item())
        ctx.save_for_backward(motion, pos, sc, rt, scratch)
        ctx.meta = (n, f, h, w, tuple(recon4), float(alpha), k)
        return tuple(o[:k] for o in outs)

    @staticmethod
    def backward(ctx, g_pos, g_sc, g_rt, g_op, g_col):
        motion, pos, sc, rt, scratch = ctx.saved_tensors
        n, f, h, w, recon4, alpha, k = ctx.meta
        dev = pos.device
        lib = _lib.lib()
        f32 = dict(device=dev, dtype=torch.float32)
        grads = [None if g is None else _f32c(g) for g in (g_pos, g_sc, g_rt, g_op, g_col)]
        d = [torch.empty((n, 2), **f32), torch.empty((n, 2), **f32), torch.empty((n,), **f32),
             torch.empty((n,), **f32), torch.empty((n, f), **f32)]
        d_motion = torch.empty(motion.shape, **f32) if ctx.needs_input_grad[0] else None
        bscratch = torch.empty((lib.oss_warp_canvas_backward_scratch_bytes(h, w),), device=dev, dtype=torch.uint8)
        recon = torch.tensor(recon4, dtype=torch.float32)
        with torch.cuda.device(dev):
            _lib.check(lib.oss_warp_canvas_backward(
                n, f, motion.shape[1], motion.shape[2], h, w, motion.data_ptr(), alpha, recon.data_ptr(),
                pos.data_ptr(), sc.data_ptr(), rt.data_ptr(), scratch.data_ptr(),
                *(None if g is None or g.numel() == 0 else g.data_ptr() for g in grads),
                *(t.data_ptr() if t.numel() else None for t in d), _lib.ptr(d_motion), bscratch.data_ptr(),
                bscratch.numel(), stream_of(pos)), "oss_warp_canvas_backward")
        return (d_motion, *d, None, None, None, None)


def _f32c(t: torch.Tensor) -> torch.Tensor:
    return aligned(t.to(dtype=torch.float32).contiguous(), 8)


def warp_canvas(canvas, motion_lr: torch.Tensor, output_hw: Tuple[int, int],
                sigma_recon: torch.Tensor | float = 0.5, alpha: float = 1.0, compact: bool = True) -> CanvasState:
    """Warp canvas positions by alpha * motion and resample covariances.

    Returns a fresh CanvasState holding the Gaussians whose warped centre
    stays inside the frame, in input order (one device->host read of the
    count, as the reference's ``.item()`` at canvas_warp.py:253).
    Differentiable in the canvas tensors and motion_lr (its first batch item,
    the one the warp reads); sigma_recon is a constant.

    compact=False (forward only) keeps every slot: a Gaussian whose centre
    leaves the frame is parked far outside it with opacity and colours 0, so a
    render of the result is the render of the compacted canvas (the same
    per-tile order of the survivors) and nothing is read on the host.
    """
    h, w = _validate_motion(motion_lr, output_hw)
    count = _validate_canvas(canvas)
    src = [canvas.positions[:count], canvas.scales[:count], canvas.rotations[:count], canvas.opacities[:count],
           canvas.colors[:count]]
    if isinstance(sigma_recon, torch.Tensor) and sigma_recon.requires_grad and torch.is_grad_enabled():
        raise RuntimeError("warp_canvas takes sigma_recon as a constant; detach it")
    if count == 0:
        return CanvasState(*(t.clone() for t in src), count=0)
    dev = canvas.positions.device
    if dev.type != "cuda" or motion_lr.device != dev:
        raise RuntimeError("warp_canvas needs canvas and motion_lr on the same CUDA device")
    if not compact:
        return _warp_parked(motion_lr, src, h, w, sigma_recon, alpha)
    out_dtypes = [t.dtype for t in src]
    with torch.cuda.device(dev):
        outs = _WarpCanvas.apply(_f32c(motion_lr[0]), *(_f32c(t) for t in src), h, w, _recon4(sigma_recon),
                                 float(alpha))
    k = int(outs[0].shape[0])
    res = [o.to(dtype=dt) for o, dt in zip(outs, out_dtypes)]
    return CanvasState(*res, count=k)


def _warp_parked(motion_lr, src, h, w, sigma_recon, alpha) -> CanvasState:
    """warp_canvas(compact=False): oss_warp_canvas_parked, forward only."""
    if torch.is_grad_enabled() and any(t.requires_grad for t in (motion_lr, *src)):
        raise RuntimeError("warp_canvas(compact=False) is forward-only; use compact=True for gradients")
    dev = src[0].device
    lib = _lib.lib()
    motion = _f32c(motion_lr[0].detach())
    pos, sc, rt, op, col = (_f32c(t.detach()) for t in src)
    n, f = int(pos.shape[0]), int(col.shape[1])
    f32 = dict(device=dev, dtype=torch.float32)
    outs = [torch.empty((n, 2), **f32), torch.empty((n, 2), **f32), torch.empty((n,), **f32),
            torch.empty((n,), **f32), torch.empty((n, f), **f32)]
    scratch = torch.empty((lib.oss_warp_canvas_scratch_bytes(n),), device=dev, dtype=torch.uint8)
    recon = torch.tensor(_recon4(sigma_recon), dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib.check(
            lib.oss_warp_canvas_parked(n, f, motion.shape[1], motion.shape[2], h, w, motion.data_ptr(), float(alpha),
                                       recon.data_ptr(), pos.data_ptr(), sc.data_ptr(), rt.data_ptr(),
                                       op.data_ptr(), col.data_ptr() if f > 0 else None,
                                       *(o.data_ptr() if o.numel() else None for o in outs), scratch.data_ptr(),
                                       scratch.numel(), stream_of(pos)),
            "oss_warp_canvas_parked",
        )
    return CanvasState(*(o.to(dtype=t.dtype) for o, t in zip(outs, src)), count=n)


def warp_positions(xy: torch.Tensor, motion: torch.Tensor, hw: Tuple[int, int],
                   alpha: float = 1.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """(new_xy, in_frame) for a motion field (2, H, W) at the frame resolution."""
    if xy.ndim != 2 or xy.shape[1] != 2:
        raise ValueError(f"xy must be (N, 2); got {tuple(xy.shape)}")
    if motion.ndim != 3 or motion.shape[0] != 2:
        raise ValueError(f"motion must be (2, H, W); got {tuple(motion.shape)}")
    h, w = int(hw[0]), int(hw[1])
    if motion.shape[1] != h or motion.shape[2] != w:
        raise ValueError(f"motion spatial dims {tuple(motion.shape[1:])} disagree with hw={hw}")
    _no_grad_inputs(xy, motion)
    n = int(xy.shape[0])
    if n == 0:
        return xy.clone(), torch.zeros((0,), dtype=torch.bool, device=xy.device)
    if xy.device.type != "cuda":
        raise RuntimeError("warp_positions needs CUDA tensors")
    p, m = _f32(xy), _f32(motion)
    lib = _lib.lib()
    with torch.cuda.device(xy.device):
        out = torch.empty((n, 2), device=xy.device, dtype=torch.float32)
        flag = torch.empty((n,), device=xy.device, dtype=torch.uint8)
        _lib.check(lib.oss_warp_positions(n, h, w, m.data_ptr(), float(alpha), p.data_ptr(), out.data_ptr(),
                                          flag.data_ptr(), stream_of(p)), "oss_warp_positions")
    return out.to(dtype=xy.dtype), flag.bool()
