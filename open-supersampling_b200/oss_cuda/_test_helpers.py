"""Kernel-by-kernel helpers (reference oss/cuda/oss_cuda/_test_helpers.py:11-16)."""

from importlib import import_module

try:
    from . import _C
except ImportError:
    _C = import_module("oss_cuda._C")


def preprocess_only(xy, scale, rot, H, W, tile_size=16):
    return _C.preprocess_only(xy, scale, rot, H, W, tile_size)


def pair_construction_only(xy, scale, rot, H, W, tile_size=16):
    return _C.pair_construction_only(xy, scale, rot, H, W, tile_size)
