"""The C-ABI library loads and exports every entry point include/*.h declares,
and its host-side argument checks reject bad input before any device work.

CPU only: no call here reaches a CUDA runtime function.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT

from oss_cuda import _lib

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols() -> list[str]:
    names = []
    for h in HEADERS:
        text = h.read_text()
        names += re.findall(r"^OSS_API\s+[\w\s\*]+?\b(oss_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "oss_render_forward" in names and "oss_tile_bin_counting_sort" in names
    assert len(names) >= 16


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_every_declared_symbol():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_abi_version_and_clean_error_state():
    lib = _lib.lib()
    assert lib.oss_abi_version() == 9


def test_rejects_tile_size_other_than_16():
    lib = _lib.lib()
    rc = lib.oss_preprocess(4, 32, 32, 8, 0, None, None, None, None, None, None, None)
    assert rc == 1
    assert lib.oss_last_error().decode() == "tile_size must be 16"


def test_rejects_bad_sizes_and_modes():
    lib = _lib.lib()
    assert lib.oss_preprocess(-1, 32, 32, 16, 0, None, None, None, None, None, None, None) == 1
    assert lib.oss_last_error().decode() == "N must be non-negative"
    assert lib.oss_preprocess(1, 1 << 40, 32, 16, 0, None, None, None, None, None, None, None) == 3
    assert lib.oss_last_error().decode() == "H exceeds int32 range"
    assert lib.oss_preprocess(1, 1 << 30, 1 << 30, 16, 0, None, None, None, None, None, None, None) == 3
    assert lib.oss_last_error().decode() == "number of tiles exceeds int32 range"
    assert lib.oss_render_prepare(1, 32, 32, 7, None, None, None, 0, None, None, None, None, None, None, None, None,
                                  None, None, None, 0, None) == 1
    assert "binning mode" in lib.oss_last_error().decode()
    assert lib.oss_render_forward(1, 65, 32, 32, None, None, None, None, None, None, None, None, None, None, None,
                                  None) == 1
    assert lib.oss_last_error().decode() == "F must be <= 64"
    assert lib.oss_full_tile_pairs(1 << 20, 1 << 12, None, None, None) == 3
    assert "full-frame" in lib.oss_last_error().decode()
    assert lib.oss_tile_bin_counting_sort(4, 0, None, None, None, None, None, 0, None) == 1
    assert lib.oss_last_error().decode() == "num_tiles must be positive"
    assert lib.oss_bin_pairs(1, 32, 32, 0, None, None, None, None, 1 << 32, None, None, None, None, None, None, 0,
                             None) == 3
    assert lib.oss_last_error().decode() == "capacity exceeds int32 range"
    assert lib.oss_bin_pairs(1, 32, 32, 0, None, None, None, None, 16, None, None, 8, 8, None, None, 0, None) == 1
    assert "overflow must be non-null" in lib.oss_last_error().decode()
    # full-frame lists need capacity >= N * tiles, checked on the host
    assert lib.oss_bin_pairs(3, 32, 32, 2, None, None, None, None, 11, None, None, 8, 8, 8, None, 0, None) == 3
    assert "capacity >= N * num_tiles" in lib.oss_last_error().decode()


def test_rejects_scratch_too_small():
    lib = _lib.lib()
    need = lib.oss_render_prepare_scratch_bytes(1000)
    assert need > 0
    rc = lib.oss_render_prepare(1000, 64, 64, 0, 8, 8, 8, 0, None, None, 8, 16, 8, 16, None, 8, 8, 8, 8, need - 1,
                                None)
    assert rc == 4 and "scratch" in lib.oss_last_error().decode()
    rc = lib.oss_render_prepare(1000, 64, 64, 0, 8, 8, 8, 0, None, None, 8, 16, 8, 16, None, 8, None, 8, 8, need,
                                None)
    assert rc == 1 and "tile_count" in lib.oss_last_error().decode()
    # packed records need 16-byte alignment and the features
    rc = lib.oss_render_prepare(1000, 64, 64, 0, 8, 8, 8, 3, None, None, 16, 16, 8, 16, 32, 8, 8, 8, 8, need, None)
    assert rc == 1 and "prec" in lib.oss_last_error().decode()
    rc = lib.oss_render_prepare(1000, 64, 64, 0, 8, 8, 8, 3, 16, None, 16, 16, 8, 16, 40, 8, 8, 8, 8, need, None)
    assert rc == 1 and "prec" in lib.oss_last_error().decode()
    assert lib.oss_tile_count_elems(100) >= 100
    bneed = lib.oss_bin_pairs_scratch_bytes(1000, 5000, 16)
    rc = lib.oss_bin_pairs(1000, 64, 64, 0, 16, 8, 8, 8, 5000, None, None, 8, 8, 8, 8, bneed - 1, None)
    assert rc == 4 and "scratch" in lib.oss_last_error().decode()
    assert lib.oss_bin_pairs(1000, 64, 64, 0, 16, 8, 8, 8, 5000, 8, None, 8, 8, 8, 8, bneed, None) == 1
    assert "sort_key and key_order" in lib.oss_last_error().decode()
    assert lib.oss_depth_order(10, 8, 8, 8, 8, lib.oss_depth_order_scratch_bytes(10) - 1, None) == 4
    assert lib.oss_alpha_pair_grad_stride(3) == 12


def test_render_bin_argument_checks():
    """The one-call binning refuses bad arguments before touching the device."""
    lib = _lib.lib()
    need = lib.oss_render_bin_scratch_bytes(1000, 5000, 16)
    assert need >= lib.oss_bin_pairs_scratch_bytes(1000, 5000, 16)

    def call(mode=0, capacity=5000, scratch_bytes=need, tile_count=8, frames=1):
        return lib.oss_render_bin(1000, 64, 64, frames, None, mode, 8, 8, 8, 0, None, None, 8, 16, 8, 16, None, 8,
                                  tile_count, 8, capacity, 8, 8, 16, scratch_bytes, None)

    assert call(scratch_bytes=need - 1) == 4 and "scratch" in lib.oss_last_error().decode()
    assert call(mode=2) == 1 and "full-frame" in lib.oss_last_error().decode()
    assert call(mode=7) == 1
    assert call(capacity=-1) == 1
    assert call(capacity=1 << 31) == 3 and "int32" in lib.oss_last_error().decode()
    assert call(tile_count=None) == 1 and "tile_count" in lib.oss_last_error().decode()
    assert call(frames=0) == 1 and "frames" in lib.oss_last_error().decode()
    assert call(frames=2) == 1 and "frame_offsets" in lib.oss_last_error().decode()
    assert call(frames=1 << 30) == 3
    assert lib.oss_render_forward_frames(1, 3, 64, 64, 0, None, None, None, None, None, None, None, None, None,
                                         None, None, None) == 1
    assert lib.oss_backward_items_frames(64, 64, -1, 0, None, None, 0, None) == 1


def test_scratch_sizes_are_monotone():
    lib = _lib.lib()
    a = lib.oss_bin_pairs_scratch_bytes(1000, 10_000, 500)
    b = lib.oss_bin_pairs_scratch_bytes(1000, 20_000, 500)
    assert 0 < a < b
    assert lib.oss_render_backward_scratch_bytes(1000, 3, 10) >= 1000 * 8 * 4 + (10 + 32) * 16
    assert lib.oss_entry_record_floats(3) == 8 and lib.oss_entry_record_floats(64) % 4 == 0
    assert lib.oss_tile_bin_counting_sort_scratch_bytes(0, 1) > 0


def test_python_checks_mirror_reference_messages():
    import torch

    from oss_cuda import _raster

    with pytest.raises(RuntimeError, match="xy must be CUDA"):
        _raster.check_gaussians(torch.zeros(3, 2), torch.zeros(3, 2), torch.zeros(3))
    with pytest.raises(RuntimeError, match="tile_size must be 16"):
        _raster.check_hw(32, 32, 8)
    with pytest.raises(ValueError):
        _raster.binning_mode("bogus")
    assert _raster.binning_mode(None) == _lib.OSS_BIN_EXACT56
    assert _raster.binning_mode(None, default="exact") == _lib.OSS_BIN_EXACT
    assert _raster.binning_mode("exact56") == _lib.OSS_BIN_EXACT56
    assert _raster.binning_mode("tight3sigma") == _lib.OSS_BIN_TIGHT3SIGMA
