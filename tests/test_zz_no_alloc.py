"""The allocation-free tile binning entry point.

oss_tile_bin_counting_sort_noalloc serves callers that cannot allocate device
memory (a per-frame hook in a host application with a fixed memory budget, or
an embedding host that owns all allocations): its scratch is a fixed array in
the library's device image.  These tests call it through the C ABI and check
that it returns exactly what the allocating entry point returns, on two calls
in a row (the second smaller than the first, so leftovers of the first call in
the shared array must not leak into the second), and that it refuses sizes
beyond its stated maximum.  This file is collected last on purpose.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_N = 262144
MAX_TILES = 65536


def _call_noalloc(tile_id: torch.Tensor, gid: torch.Tensor, num_tiles: int):
    from oss_cuda import _lib

    lib = _lib.lib()
    n = tile_id.numel()
    sorted_gid = torch.full((n,), -7, device=tile_id.device, dtype=torch.int32)
    offsets = torch.full((num_tiles + 1,), -7, device=tile_id.device, dtype=torch.int32)
    rc = lib.oss_tile_bin_counting_sort_noalloc(n, num_tiles, tile_id.data_ptr(), gid.data_ptr(),
                                                sorted_gid.data_ptr(), offsets.data_ptr(),
                                                torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "oss_tile_bin_counting_sort_noalloc")
    return sorted_gid, offsets


def test_noalloc_matches_allocating_entry_point(cuda_device):
    from oss_cuda import tile_bin_counting_sort

    for seed, n, num_tiles in ((11, MAX_N, MAX_TILES), (12, 5000, 37)):
        rng = np.random.default_rng(seed)
        tile_id = torch.from_numpy(rng.integers(-2, num_tiles + 2, size=n).astype(np.int32)).to(cuda_device)
        gid = torch.from_numpy(rng.integers(0, 1 << 30, size=n).astype(np.int32)).to(cuda_device)
        got_gid, got_offs = _call_noalloc(tile_id, gid, num_tiles)
        ref_gid, ref_offs = tile_bin_counting_sort(tile_id, gid, num_tiles)
        torch.cuda.synchronize()
        assert torch.equal(got_offs, ref_offs)
        assert torch.equal(got_gid, ref_gid)


def test_noalloc_rejects_sizes_beyond_its_maximum(cuda_device):
    from oss_cuda import _lib

    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.oss_tile_bin_counting_sort_noalloc(MAX_N + 1, 16, None, None, None, None, stream) == 3
    assert "no-alloc maximum" in lib.oss_last_error().decode()
    assert lib.oss_tile_bin_counting_sort_noalloc(16, MAX_TILES + 1, None, None, None, None, stream) == 3
    assert "no-alloc maximum" in lib.oss_last_error().decode()


def test_noalloc_leaves_device_memory_untouched(cuda_device):
    """After the first call in this context (which may load the library's device
    code), further calls change neither the device's free memory nor torch's
    allocator: the scratch really is the fixed array."""
    from oss_cuda import _lib

    lib = _lib.lib()
    n, num_tiles = 100_000, 8160
    rng = np.random.default_rng(13)
    tile_id = torch.from_numpy(rng.integers(0, num_tiles, size=n).astype(np.int32)).to(cuda_device)
    gid = torch.arange(n, device=cuda_device, dtype=torch.int32)
    sorted_gid = torch.empty((n,), device=cuda_device, dtype=torch.int32)
    offsets = torch.empty((num_tiles + 1,), device=cuda_device, dtype=torch.int32)
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        rc = lib.oss_tile_bin_counting_sort_noalloc(n, num_tiles, tile_id.data_ptr(), gid.data_ptr(),
                                                    sorted_gid.data_ptr(), offsets.data_ptr(), stream)
        _lib.check(rc, "oss_tile_bin_counting_sort_noalloc")

    call()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(cuda_device)[0]
    torch_bytes0 = torch.cuda.memory_allocated(cuda_device)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda_device)[0] == free0
    assert torch.cuda.memory_allocated(cuda_device) == torch_bytes0
