"""Host-side mirrors of the reference's rasterizer callers, on the B200 kernels:
canvas warp (oss/sr/v6/canvas_warp.py, oss/gaussian/canvas/warp.py), the v6
rasterizer front-end (oss/sr/v6/rasterizer.py) and the persistent canvas's
per-frame lifecycle (oss/gaussian/canvas/) and the v7 N-D time-slice rasterizer
(oss/sr/v7/nd_rasterizer.py), and the Analytic-Splatting pixel integral
(oss/sr/v6/aa_analytic_splat.py)."""

from .analytic import analytic_pixel_integral, logistic_cdf
from .canvas import CanvasState
from .v6 import V6Rasterizer, phase_feather_mask, render, render_canvas_at_lr, render_overlapped
from .nd import NDGaussian, render_nd_time_slice, time_marginal
from .persistent_canvas import (CanvasStats, GaussianBatch, PersistentCanvas, PrunePolicy, apply_prune_spawn,
                                gaussians_error_from_tiles, per_tile_mse, per_tile_mse_lr, select_for_pruning,
                                select_spawn_tiles)
from .warp import warp_canvas, warp_positions

__all__ = ["CanvasState", "CanvasStats", "GaussianBatch", "NDGaussian", "PersistentCanvas", "PrunePolicy",
           "V6Rasterizer", "analytic_pixel_integral", "logistic_cdf", "render_nd_time_slice", "time_marginal",
           "apply_prune_spawn", "gaussians_error_from_tiles", "per_tile_mse", "per_tile_mse_lr", "phase_feather_mask",
           "render", "render_canvas_at_lr", "render_overlapped", "select_for_pruning", "select_spawn_tiles",
           "warp_canvas", "warp_positions"]
