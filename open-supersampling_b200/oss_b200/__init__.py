"""Host-side mirrors of the reference's rasterizer callers, on the B200 kernels:
canvas warp (oss/sr/v6/canvas_warp.py, oss/gaussian/canvas/warp.py) and the
v6 rasterizer front-end (oss/sr/v6/rasterizer.py)."""

from .canvas import CanvasState
from .warp import warp_canvas, warp_positions

__all__ = ["CanvasState", "warp_canvas", "warp_positions"]
