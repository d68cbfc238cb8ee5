"""B200 (sm_100a) drop-in for the reference's ``oss_cuda`` package
(reference oss/cuda/oss_cuda/__init__.py:1-10)."""

from ._raster import pair_capacity_overflowed
from .attention import fused_window_cross_attention
from .rasterizer import rasterize_gaussians
from .tile_bin import tile_bin_counting_sort

__all__ = [
    "rasterize_gaussians",
    "fused_window_cross_attention",
    "tile_bin_counting_sort",
    "pair_capacity_overflowed",
]
__version__ = "0.3.0+b200"
