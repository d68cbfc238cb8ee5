"""Canvas SoA contract (reference oss/sr/v6/model.py:977-990)."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class CanvasState:
    positions: torch.Tensor  # (N, 2) pixel centres (x, y)
    scales: torch.Tensor     # (N, 2) principal-axis scales
    rotations: torch.Tensor  # (N,) radians
    opacities: torch.Tensor  # (N,)
    colors: torch.Tensor     # (N, F)
    count: int
