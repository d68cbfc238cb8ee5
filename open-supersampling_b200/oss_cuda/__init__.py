"""B200 (sm_100a) drop-in for the reference's ``oss_cuda`` package
(reference oss/cuda/oss_cuda/__init__.py:1-10)."""

from ._raster import pair_capacity_overflowed
from .attention import fused_window_cross_attention
from .rasterizer import rasterize_gaussians, rasterize_gaussians_batched
from .tile_bin import tile_bin_counting_sort


def warp_canvas_cuda(canvas, motion_lr, output_hw, sigma_recon=0.5, alpha=1.0):
    """GS-STVSR canvas warp at extrapolation alpha on the B200 kernels
    (oss/sr/v6/canvas_warp.py:177-254 with the motion scaled by alpha)."""
    from oss_b200.warp import warp_canvas

    return warp_canvas(canvas, motion_lr, output_hw, sigma_recon=sigma_recon, alpha=alpha)


__all__ = [
    "rasterize_gaussians",
    "rasterize_gaussians_batched",
    "warp_canvas_cuda",
    "fused_window_cross_attention",
    "tile_bin_counting_sort",
    "pair_capacity_overflowed",
]
__version__ = "0.3.0+b200"
