"""Tile binning helper backed by the B200 C-ABI library.

Drop-in for reference oss/cuda/oss_cuda/tile_bin.py:22-40.  The sort is a
stable counting sort: within a tile, gids keep their input order (the
reference's atomic cursor leaves that order unspecified).
"""
from __future__ import annotations

from importlib import import_module

import torch

try:
    from . import _C

    _COMPILED = True
except ImportError:
    try:
        _C = import_module("oss_cuda._C")
        _COMPILED = True
    except ImportError:
        _C = None
        _COMPILED = False


def tile_bin_counting_sort(
    tile_id: torch.Tensor, gid: torch.Tensor, num_tiles: int
) -> tuple[torch.Tensor, torch.Tensor]:
    """Group ``gid`` values by ``tile_id`` using a device counting sort.

    Returns ``(sorted_gid, tile_offsets)``. Values for tile ``t`` occupy
    ``sorted_gid[tile_offsets[t]:tile_offsets[t + 1]]``.
    """
    if not _COMPILED:
        raise RuntimeError(
            "oss_cuda extension not compiled. Run: python open-supersampling_b200/build.py"
        )
    if not tile_id.is_cuda or not gid.is_cuda:
        raise RuntimeError("tile_id and gid must be CUDA tensors")
    return _C.tile_bin_counting_sort(
        tile_id.contiguous().to(torch.int32),
        gid.contiguous().to(torch.int32),
        int(num_tiles),
    )
