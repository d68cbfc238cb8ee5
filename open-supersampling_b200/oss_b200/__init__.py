"""Host-side mirrors of the reference's rasterizer callers, on the B200 kernels:
canvas warp (oss/sr/v6/canvas_warp.py, oss/gaussian/canvas/warp.py) and the
v6 rasterizer front-end (oss/sr/v6/rasterizer.py)."""

from .canvas import CanvasState
from .v6 import V6Rasterizer, phase_feather_mask, render, render_canvas_at_lr, render_overlapped
from .warp import warp_canvas, warp_positions

__all__ = ["CanvasState", "V6Rasterizer", "phase_feather_mask", "render", "render_canvas_at_lr", "render_overlapped",
           "warp_canvas", "warp_positions"]
