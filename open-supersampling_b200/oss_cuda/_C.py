"""Drop-in for the reference's compiled ``oss_cuda._C`` module.

Same entry points, argument order, return tuples and error messages as
reference oss/cuda/src/bindings.cpp:65-78, implemented over the C ABI of
liboss_b200.so.  Importing this module raises ImportError when the library is
not built, exactly like a missing pybind extension, so the package's
``_COMPILED`` gate behaves as in the reference (oss_cuda/rasterizer.py:10-21).
"""
from __future__ import annotations

import torch

from . import _lib
from ._raster import (
    INT32_MAX,
    aligned,
    bin_gaussians,
    binning_mode,
    check_float_cuda,
    check_gaussians,
    check_hw,
    check_int_cuda,
    render_forward,
    stream_of,
)

if not _lib.available():
    raise ImportError(f"liboss_b200.so not loadable: {_lib.load_error()}")


def rasterize_forward(xy, scale, rot, feat, h, w, tile_size=16, topk_norm=True, *, binning=None):
    """(out[F,H,W], gaussian_idx_sorted[P], tile_offsets[T+1], conic[N,3]).

    Reference: rasterizer_fwd.cu:478-590.  ``topk_norm`` is accepted and
    ignored, as in the reference (:488).  ``binning`` selects the tile lists:
    "exact56" (default: the reference's full-tail image to within 6.9e-13 per
    unit of feature left out), "exact" (every nonzero fp32 weight), "full" (the
    reference's literal full-frame lists) or "tight3sigma".
    """
    del topk_norm
    h, w, tile_size = int(h), int(w), int(tile_size)
    n, _ = check_gaussians(xy, scale, rot, feat)
    check_hw(h, w, tile_size)
    mode = binning_mode(binning)
    with torch.cuda.device(xy.device):
        b = bin_gaussians(xy, scale, rot, h, w, mode, feat=feat)
        out = render_forward(b, aligned(feat, 4), None)
    return out, b.gid_sorted, b.tile_offsets, b.conic


def rasterize_backward(xy, scale, rot, feat, conic, gaussian_idx_sorted, tile_offsets, grad_out, h, w, tile_size=16):
    """(d_xy[N,2], d_conic[N,3], d_feat[N,F]) for caller-supplied lists.

    Reference: rasterizer_bwd.cu:157-247.  Works for any lists (per-pair
    partials, then fp32 atomics); the autograd path uses the deterministic
    backward instead.
    """
    for t, name in ((xy, "xy"), (scale, "scale"), (rot, "rot"), (feat, "feat"), (conic, "conic"),
                    (grad_out, "grad_out")):
        check_float_cuda(t, name)
    check_int_cuda(gaussian_idx_sorted, "gaussian_idx_sorted")
    check_int_cuda(tile_offsets, "tile_offsets")
    if xy.dim() != 2 or xy.size(1) != 2:
        raise RuntimeError("xy must be (N,2)")
    if scale.dim() != 2 or scale.size(1) != 2:
        raise RuntimeError("scale must be (N,2)")
    if rot.dim() != 1:
        raise RuntimeError("rot must be (N,)")
    if feat.dim() != 2:
        raise RuntimeError("feat must be (N,F)")
    if conic.dim() != 2 or conic.size(1) != 3:
        raise RuntimeError("conic must be (N,3)")
    if gaussian_idx_sorted.dim() != 1:
        raise RuntimeError("gaussian_idx_sorted must be 1D")
    if tile_offsets.dim() != 1:
        raise RuntimeError("tile_offsets must be 1D")
    if grad_out.dim() != 3:
        raise RuntimeError("grad_out must be (F,H,W)")
    n = int(xy.size(0))
    for t, name in ((scale, "scale"), (rot, "rot"), (feat, "feat"), (conic, "conic")):
        if t.size(0) != n:
            raise RuntimeError(f"xy/{name} N mismatch")
    h, w, tile_size = int(h), int(w), int(tile_size)
    ntx, nty, num_tiles, _ = check_hw(h, w, tile_size)
    f = int(feat.size(1))
    if f > _lib.MAX_CHANNELS:
        raise RuntimeError("F must be <= 64")
    if tuple(grad_out.shape) != (f, h, w):
        raise RuntimeError("grad_out shape mismatch: expected (F,H,W)")
    if tile_offsets.size(0) != num_tiles + 1:
        raise RuntimeError("tile_offsets length mismatch")
    lib = _lib.lib()
    dev = xy.device
    with torch.cuda.device(dev):
        f32 = dict(device=dev, dtype=torch.float32)
        d_xy = torch.empty((n, 2), **f32)
        d_conic = torch.empty((n, 3), **f32)
        d_feat = torch.empty((n, f), **f32)
        total = int(gaussian_idx_sorted.numel())
        nbytes = lib.oss_rasterize_backward_lists_scratch_bytes(n, total, num_tiles)
        scratch = torch.empty((max(1, nbytes),), device=dev, dtype=torch.uint8)
        xy_a = aligned(xy, 8)
        _lib.check(
            lib.oss_rasterize_backward_lists(n, f, h, w, xy_a.data_ptr(), conic.data_ptr(), feat.data_ptr(),
                                             gaussian_idx_sorted.data_ptr(), total, tile_offsets.data_ptr(),
                                             grad_out.data_ptr(), d_xy.data_ptr(), d_conic.data_ptr(),
                                             d_feat.data_ptr(), scratch.data_ptr(), scratch.numel(), stream_of(xy)),
            "rasterize_backward",
        )
    return d_xy, d_conic, d_feat


def conic_to_scale_rot_grad(scale, rot, d_conic):
    """(d_scale[N,2], d_rot[N]).  Reference: rasterizer_bwd.cu:249-289."""
    check_float_cuda(scale, "scale")
    check_float_cuda(rot, "rot")
    check_float_cuda(d_conic, "d_conic")
    if scale.dim() != 2 or scale.size(1) != 2:
        raise RuntimeError("scale must be (N,2)")
    if rot.dim() != 1:
        raise RuntimeError("rot must be (N,)")
    if d_conic.dim() != 2 or d_conic.size(1) != 3:
        raise RuntimeError("d_conic must be (N,3)")
    if scale.size(0) != rot.size(0):
        raise RuntimeError("scale/rot N mismatch")
    if scale.size(0) != d_conic.size(0):
        raise RuntimeError("scale/d_conic N mismatch")
    n = int(scale.size(0))
    if n > INT32_MAX:
        raise RuntimeError("N exceeds int32 range")
    lib = _lib.lib()
    with torch.cuda.device(scale.device):
        d_scale = torch.zeros((n, 2), device=scale.device, dtype=torch.float32)
        d_rot = torch.zeros((n,), device=scale.device, dtype=torch.float32)
        _lib.check(
            lib.oss_conic_to_scale_rot_grad(n, aligned(scale, 8).data_ptr(), rot.data_ptr(), d_conic.data_ptr(),
                                            d_scale.data_ptr(), d_rot.data_ptr(), stream_of(scale)),
            "conic_to_scale_rot_grad",
        )
    return d_scale, d_rot


def preprocess_only(xy, scale, rot, h, w, tile_size=16):
    """(conic[N,3], aabb[N,4] int32 (tx0,ty0,tx1,ty1), pair_count[N] int32).

    Reference: rasterizer_fwd.cu:325-379 (tight-ellipse AABB, tau = 9).
    """
    h, w, tile_size = int(h), int(w), int(tile_size)
    n, _ = check_gaussians(xy, scale, rot)
    check_hw(h, w, tile_size)
    lib = _lib.lib()
    dev = xy.device
    with torch.cuda.device(dev):
        conic = torch.empty((n, 3), device=dev, dtype=torch.float32)
        aabb = torch.empty((n, 4), device=dev, dtype=torch.int32)
        pair_count = torch.empty((n,), device=dev, dtype=torch.int32)
        if n == 0:
            return conic, aabb, pair_count
        _lib.check(
            lib.oss_preprocess(n, h, w, tile_size, _lib.OSS_BIN_TIGHT3SIGMA, aligned(xy, 8).data_ptr(),
                               aligned(scale, 8).data_ptr(), rot.data_ptr(), conic.data_ptr(), aabb.data_ptr(),
                               pair_count.data_ptr(), stream_of(xy)),
            "preprocess_only",
        )
    return conic, aabb, pair_count


def pair_construction_only(xy, scale, rot, h, w, tile_size=16):
    """(gid_sorted[P], tile_offsets[T+1], conic[N,3], total_pairs int).

    Reference: rasterizer_fwd.cu:381-476 (3-sigma lists sorted by
    (tile << 32 | gid)); here a deterministic counting sort gives the same order.
    """
    h, w, tile_size = int(h), int(w), int(tile_size)
    check_gaussians(xy, scale, rot)
    check_hw(h, w, tile_size)
    with torch.cuda.device(xy.device):
        b = bin_gaussians(xy, scale, rot, h, w, _lib.OSS_BIN_TIGHT3SIGMA)
    return b.gid_sorted, b.tile_offsets, b.conic, b.total_pairs


def tile_bin_counting_sort(tile_id, gid, num_tiles):
    """(sorted_gid[n], tile_offsets[T+1]).  Reference: tile_bin_counting_sort.cu:71-128."""
    for t, name in ((tile_id, "tile_id"), (gid, "gid")):
        check_int_cuda(t, name)
        if t.dim() != 1:
            raise RuntimeError(f"{name} must be 1D")
    if tile_id.numel() != gid.numel():
        raise RuntimeError("tile_id and gid must have the same length")
    num_tiles = int(num_tiles)
    if num_tiles <= 0:
        raise RuntimeError("num_tiles must be positive")
    if num_tiles > INT32_MAX:
        raise RuntimeError("num_tiles exceeds int32 range")
    n = int(tile_id.numel())
    if n > INT32_MAX:
        raise RuntimeError("N exceeds int32 range")
    lib = _lib.lib()
    dev = tile_id.device
    with torch.cuda.device(dev):
        sorted_gid = torch.empty((n,), device=dev, dtype=torch.int32)
        tile_offsets = torch.empty((num_tiles + 1,), device=dev, dtype=torch.int32)
        nbytes = lib.oss_tile_bin_counting_sort_scratch_bytes(n, num_tiles)
        scratch = torch.empty((max(1, nbytes),), device=dev, dtype=torch.uint8)
        _lib.check(
            lib.oss_tile_bin_counting_sort(n, num_tiles, tile_id.data_ptr(), gid.data_ptr(), sorted_gid.data_ptr(),
                                           tile_offsets.data_ptr(), scratch.data_ptr(), scratch.numel(),
                                           stream_of(tile_id)),
            "tile_bin_counting_sort",
        )
    return sorted_gid, tile_offsets
