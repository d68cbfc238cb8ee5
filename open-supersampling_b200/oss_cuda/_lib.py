"""ctypes binding of liboss_b200.so, the C ABI declared in include/oss_raster.h.

Loading is strict: if the shared library is missing or fails to load, every
op raises.  There is no CPU or PyTorch fallback on the product path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "liboss_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

OSS_OK = 0
OSS_BIN_TIGHT3SIGMA = 0
OSS_BIN_EXACT = 1
OSS_BIN_FULL = 2
OSS_BIN_EXACT56 = 3
BINNING_MODES = {"tight3sigma": OSS_BIN_TIGHT3SIGMA, "exact": OSS_BIN_EXACT, "full": OSS_BIN_FULL,
                 "exact56": OSS_BIN_EXACT56}
# the binning of the reference-signature call: its image is the reference's full-tail sum to within
# 6.9e-13 per unit of feature left out (every weight left out is below e^-28)
DEFAULT_BINNING = "exact56"
TILE = 16
MAX_CHANNELS = 64

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_p = ctypes.c_void_p

# name -> (restype, argtypes); must match include/oss_raster.h
SIGNATURES = {
    "oss_last_error": (ctypes.c_char_p, []),
    "oss_abi_version": (ctypes.c_int, []),
    "oss_preprocess": (ctypes.c_int, [_i64, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _p]),
    "oss_render_prepare_scratch_bytes": (_i64, [_i64]),
    "oss_tile_count_elems": (_i64, [_i64]),
    "oss_render_prepare": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i32, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_bin_pairs_scratch_bytes": (_i64, [_i64, _i64, _i64]),
    "oss_bin_pairs": (
        ctypes.c_int, [_i64, _i64, _i64, _i32, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_render_bin_scratch_bytes": (_i64, [_i64, _i64, _i64]),
    "oss_render_bin": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _p, _i32, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p,
         _p, _i64, _p]),
    "oss_publish_total": (ctypes.c_int, [_p, _p, _p]),
    "oss_depth_order_scratch_bytes": (_i64, [_i64]),
    "oss_depth_order": (ctypes.c_int, [_i64, _p, _p, _p, _p, _i64, _p]),
    "oss_render_alpha_forward": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_alpha_pair_grad_stride": (ctypes.c_int, [_i64]),
    "oss_render_alpha_backward_scratch_bytes": (_i64, [_i64, _i64]),
    "oss_render_alpha_backward": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
         _p, _i64, _p],
    ),
    "oss_entry_record_floats": (ctypes.c_int, [_i64]),
    "oss_render_forward": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_render_forward_frames": (
        ctypes.c_int, [_i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_render_backward_scratch_bytes": (_i64, [_i64, _i64, _i64]),
    "oss_render_backward": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
         _i64, _p],
    ),
    "oss_pair_grad_stride": (ctypes.c_int, [_i64]),
    "oss_backward_items": (ctypes.c_int, [_i64, _i64, _i64, _p, _p, _i64, _p]),
    "oss_backward_items_frames": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _i64, _p]),
    "oss_render_backward_items_frames": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_render_backward_items": (
        ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_render_backward_pairs_scratch_bytes": (_i64, [_i64, _i64]),
    "oss_render_backward_pairs": (
        ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_reduce_pair_grads": (ctypes.c_int, [_i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_rasterize_backward_lists_scratch_bytes": (_i64, [_i64, _i64, _i64]),
    "oss_rasterize_backward_lists": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _p],
    ),
    "oss_make_geo": (ctypes.c_int, [_i64, _p, _p, _p, _p]),
    "oss_conic_to_scale_rot_grad": (ctypes.c_int, [_i64, _p, _p, _p, _p, _p, _p]),
    "oss_full_tile_pairs": (ctypes.c_int, [_i64, _i64, _p, _p, _p]),
    "oss_warp_canvas_scratch_bytes": (_i64, [_i64]),
    "oss_warp_canvas_parked": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _i64, _i64, _p, ctypes.c_float, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
         _i64, _p],
    ),
    "oss_warp_canvas": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _i64, _i64, _p, ctypes.c_float, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
         _p, _i64, _p],
    ),
    "oss_v6_sanitize": (ctypes.c_int, [_i64, _i64, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                       _p]),
    "oss_v6_sanitize_backward": (ctypes.c_int, [_i64, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_warp_canvas_backward_scratch_bytes": (_i64, [_i64, _i64]),
    "oss_warp_canvas_backward": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _i64, _i64, _p, ctypes.c_float, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
         _p, _p, _p, _i64, _p]),
    "oss_warp_positions": (ctypes.c_int, [_i64, _i64, _i64, _p, ctypes.c_float, _p, _p, _p, _p]),
    "oss_analytic_pixel_integral": (ctypes.c_int, [_i64, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_analytic_pixel_integral_backward": (ctypes.c_int, [_i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                                            _p, _p]),
    "oss_logistic_cdf": (ctypes.c_int, [_i64, _p, _p, _p, _p]),
    "oss_render_analytic_forward": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p]),
    "oss_render_analytic_backward_scratch_bytes": (_i64, [_i64, _i64]),
    "oss_render_analytic_backward": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p,
                                                    _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_nd_record_floats": (_i64, [_i64]),
    "oss_nd_condition": (ctypes.c_int, [_i64, _i64, _i64, _p, _p, _p, ctypes.c_float, _i32, ctypes.c_float,
                                        ctypes.c_float, _p, _p, _p, _p, _p]),
    "oss_nd_condition_backward": (ctypes.c_int, [_i64, _p, _p, _p, ctypes.c_float, _i32, ctypes.c_float,
                                                 ctypes.c_float, _p, _p, _p, _p, _p, _p, _p]),
    "oss_nd_prepare": (ctypes.c_int, [_i64, _i64, _i64, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
                                      _p]),
    "oss_nd_forward": (ctypes.c_int, [_i64, _i64, _i64, _p, _p, _p, _p, _p, _p]),
    "oss_nd_backward_pairs": (ctypes.c_int, [_i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_tile_mse": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _p]),
    "oss_canvas_error": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_prune_scratch_bytes": (_i64, [_i64]),
    "oss_select_for_pruning": (
        ctypes.c_int,
        [_i64, _p, _p, _p, _p, _i64, _i64, ctypes.c_double, ctypes.c_double, _i64, ctypes.c_double, _p, _p, _p, _p,
         _i64, _p]),
    "oss_spawn_tiles_scratch_bytes": (_i64, [_i64]),
    "oss_select_spawn_tiles": (ctypes.c_int, [_i64, _i64, _p, _p, _i64, _p, _p, _p, _i64, _p]),
    "oss_prune_spawn_scratch_bytes": (_i64, [_i64]),
    "oss_apply_prune_spawn": (
        ctypes.c_int,
        [_i64, _i64, _p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_feather_supported": (ctypes.c_int, [_i32, _i64, _i64, _i64]),
    "oss_feather_virtual_count": (_i64, [_i64]),
    "oss_render_prepare_feathered_scratch_bytes": (_i64, [_i64]),
    "oss_render_prepare_feathered": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i32, _i32, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_render_forward_feathered": (ctypes.c_int, [_i64, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_render_backward_feathered": (
        ctypes.c_int, [_i64, _i64, _i64, _i64, _i32, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "oss_reduce_pair_grads_feathered": (
        ctypes.c_int, [_i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "oss_tile_bin_counting_sort_noalloc": (ctypes.c_int, [_i64, _i64, _p, _p, _p, _p, _p]),
    "oss_tile_bin_counting_sort_scratch_bytes": (_i64, [_i64, _i64]),
    "oss_tile_bin_counting_sort": (ctypes.c_int, [_i64, _i64, _p, _p, _p, _p, _p, _i64, _p]),
}

_LIB = None
_LOAD_ERROR: str | None = None


def _load():
    global _LIB, _LOAD_ERROR
    if _LIB is not None or _LOAD_ERROR is not None:
        return _LIB
    path = os.environ.get("OSS_B200_LIB", str(LIB_PATH))
    try:
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    except OSError as exc:  # missing or unloadable .so
        _LOAD_ERROR = f"{path}: {exc}"
    except AttributeError as exc:  # stale .so without a symbol
        _LOAD_ERROR = f"{path}: missing symbol ({exc})"
    return _LIB


def available() -> bool:
    return _load() is not None


def load_error() -> str | None:
    _load()
    return _LOAD_ERROR


def lib():
    """The loaded library; raises RuntimeError if it is not built."""
    handle = _load()
    if handle is None:
        raise RuntimeError(
            "oss_cuda extension not compiled (liboss_b200.so failed to load: "
            f"{_LOAD_ERROR}). Run: python open-supersampling_b200/build.py"
        )
    return handle


def check(rc: int, what: str) -> None:
    if rc != OSS_OK:
        msg = lib().oss_last_error().decode("utf-8", "replace")
        raise RuntimeError(f"{what}: {msg} (status {rc})")


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for an absent optional operand)."""
    if t is None:
        return None
    return t.data_ptr()
