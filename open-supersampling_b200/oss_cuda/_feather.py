"""Host orchestration of the one-pass feathered overlapping-tile render over the
C ABI (csrc/feather.cu): the reference's V6Rasterizer._render_overlapped
(oss/sr/v6/rasterizer.py:159-242) as one render of up to four virtual
Gaussians per Gaussian, each with its separable feather window.

prepare_feathered -> (one host read of the pair total, unless a capacity is
given) -> bin over the 4N virtual Gaussians -> forward with the window; the
backward reuses the lists and the forward's entry records and patterns, and
the reduce sums each Gaussian's variants.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch.autograd import Function

from . import _lib
from ._raster import INT32_MAX, aligned, check_hw, read_total, sticky_overflow, stream_of


def supported(overlap: int, f: int, h: int, w: int) -> bool:
    """Whether the one-pass path takes this call (F <= 16, tiles per axis within
    int16, an overlap whose weight sum stays clear of the reference's 1e-6 clamp)."""
    return bool(_lib.lib().oss_feather_supported(int(overlap), int(f), int(h), int(w)))


@dataclass
class FeatherBinned:
    n: int
    h: int
    w: int
    overlap: int
    conic: torch.Tensor         # (N, 3)
    geo: torch.Tensor           # (N, 8)
    vaabb: torch.Tensor         # (4N, 4) int32 tile hulls of the virtual Gaussians
    vpair_offset: torch.Tensor  # (4N + 1,) int32
    vprec: torch.Tensor         # (4N, record floats) packed forward records
    vwin: torch.Tensor          # (4N, 4) int32 packed phase ranges
    total_pairs: int
    gid_sorted: torch.Tensor
    tile_offsets: torch.Tensor


def bin_feathered(xy, scale, rot, feat, opacity, h, w, mode, overlap, capacity=None) -> FeatherBinned:
    lib = _lib.lib()
    n, f = int(xy.size(0)), int(feat.size(1))
    _, _, num_tiles, _ = check_hw(h, w, _lib.TILE)
    nv = int(lib.oss_feather_virtual_count(n))
    dev = xy.device
    xy, scale, feat = aligned(xy, 8), aligned(scale, 8), aligned(feat, 4)
    stream = stream_of(xy)
    f32 = dict(device=dev, dtype=torch.float32)
    i32 = dict(device=dev, dtype=torch.int32)
    conic = torch.empty((n, 3), **f32)
    geo = torch.empty((n, 8), **f32)
    vaabb = torch.empty((nv, 4), **i32)
    vpair_offset = torch.empty((nv + 1,), **i32)
    vprec = torch.empty((nv, lib.oss_entry_record_floats(f)), **f32)
    vwin = torch.empty((nv, 4), **i32)
    total = torch.empty((1,), device=dev, dtype=torch.int64)
    tile_count = torch.empty((max(1, lib.oss_tile_count_elems(num_tiles)),), **i32)
    tile_offsets = torch.empty((num_tiles + 1,), **i32)
    scratch = torch.empty((max(8, lib.oss_render_prepare_feathered_scratch_bytes(n)),), device=dev, dtype=torch.uint8)
    _lib.check(lib.oss_render_prepare_feathered(
        n, h, w, mode, int(overlap), xy.data_ptr(), scale.data_ptr(), rot.data_ptr(), f, feat.data_ptr(),
        _lib.ptr(opacity), conic.data_ptr(), geo.data_ptr(), vaabb.data_ptr(), vpair_offset.data_ptr(),
        vprec.data_ptr(), vwin.data_ptr(), total.data_ptr(), tile_count.data_ptr(), tile_offsets.data_ptr(),
        scratch.data_ptr(), scratch.numel(), stream), "oss_render_prepare_feathered")
    total_pairs = int(capacity) if capacity is not None else read_total(total, stream)
    if total_pairs > INT32_MAX:
        raise RuntimeError("total pair count exceeds int32 range")
    gid_sorted = torch.empty((max(1, total_pairs),), **i32)
    overflow = torch.empty((1,), **i32)
    scratch2 = torch.empty((max(1, lib.oss_bin_pairs_scratch_bytes(nv, total_pairs, num_tiles)),), device=dev,
                           dtype=torch.uint8)
    # the virtual Gaussians' lists follow their hulls (list mode, whatever the box mode was)
    _lib.check(lib.oss_bin_pairs(nv, h, w, _lib.OSS_BIN_TIGHT3SIGMA, vaabb.data_ptr(), vpair_offset.data_ptr(),
                                 tile_count.data_ptr(), total.data_ptr(), total_pairs, None, None,
                                 gid_sorted.data_ptr(), tile_offsets.data_ptr(), overflow.data_ptr(),
                                 scratch2.data_ptr(), scratch2.numel(), stream), "oss_bin_pairs")
    if capacity is not None:
        sticky_overflow(dev).bitwise_or_(overflow)
    return FeatherBinned(n, h, w, int(overlap), conic, geo, vaabb, vpair_offset, vprec, vwin, total_pairs,
                         gid_sorted, tile_offsets)


def forward(b: FeatherBinned, f: int, records: bool):
    lib = _lib.lib()
    dev = b.geo.device
    image = torch.empty((f, b.h, b.w), device=dev, dtype=torch.float32)
    rec = pat = None
    if records and b.total_pairs > 0:
        rec = torch.empty((b.total_pairs, lib.oss_entry_record_floats(f)), device=dev, dtype=torch.float32)
        pat = torch.empty((b.total_pairs,), device=dev, dtype=torch.int16)
    _lib.check(lib.oss_render_forward_feathered(
        int(b.vpair_offset.numel()) - 1, f, b.h, b.w, b.overlap, b.vprec.data_ptr(), b.vwin.data_ptr(),
        b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(), image.data_ptr(), _lib.ptr(rec), _lib.ptr(pat),
        stream_of(image)), "oss_render_forward_feathered")
    return image, rec, pat


def backward(b: FeatherBinned, feat, opacity, scale, rot, grad, rec, pat):
    lib = _lib.lib()
    dev = feat.device
    n, f = b.n, int(feat.size(1))
    f32 = dict(device=dev, dtype=torch.float32)
    d_xy, d_conic, d_feat = torch.empty((n, 2), **f32), torch.empty((n, 3), **f32), torch.empty((n, f), **f32)
    d_opacity = torch.empty((n,), **f32) if opacity is not None else None
    d_scale, d_rot = torch.empty((n, 2), **f32), torch.empty((n,), **f32)
    num_tiles = int(b.tile_offsets.numel()) - 1
    nv = int(b.vpair_offset.numel()) - 1
    stream = stream_of(feat)
    stride = lib.oss_pair_grad_stride(f)
    pg_bytes = ((max(1, b.total_pairs) * stride * 4 + 255) // 256) * 256
    items_bytes = lib.oss_render_backward_pairs_scratch_bytes(b.total_pairs, num_tiles)
    scratch = torch.empty((pg_bytes + max(16, items_bytes),), device=dev, dtype=torch.uint8)
    items = scratch.data_ptr() + pg_bytes
    if b.total_pairs > 0 and rec is not None:
        _lib.check(lib.oss_backward_items(b.h, b.w, b.total_pairs, b.tile_offsets.data_ptr(), items, items_bytes,
                                          stream), "oss_backward_items")
        _lib.check(lib.oss_render_backward_feathered(
            nv, f, b.h, b.w, b.overlap, b.vaabb.data_ptr(), b.vpair_offset.data_ptr(), b.total_pairs,
            b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(), rec.data_ptr(), pat.data_ptr(), grad.data_ptr(),
            scratch.data_ptr(), items, items_bytes, stream), "oss_render_backward_feathered")
    scale = aligned(scale, 8)
    _lib.check(lib.oss_reduce_pair_grads_feathered(
        n, f, scratch.data_ptr() if b.total_pairs > 0 else None, b.vpair_offset.data_ptr(), b.geo.data_ptr(),
        feat.data_ptr(), _lib.ptr(opacity), scale.data_ptr(), rot.data_ptr(), d_xy.data_ptr(), d_conic.data_ptr(),
        d_feat.data_ptr(), _lib.ptr(d_opacity), d_scale.data_ptr(), d_rot.data_ptr(), stream),
        "oss_reduce_pair_grads_feathered")
    return d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot


class RasterizeFeathered(Function):
    """rasterize_gaussians(..., overlap=o) in one pass (blend="sum")."""

    @staticmethod
    def forward(ctx, xy, scale, rot, feat, opacity, h, w, mode, overlap, capacity):
        f = int(feat.size(1))
        with torch.cuda.device(xy.device):
            b = bin_feathered(xy, scale, rot, feat, opacity, h, w, mode, overlap, capacity)
            image, rec, pat = forward(b, f, records=any(ctx.needs_input_grad[:5]))
        ctx.save_for_backward(scale, rot, feat, opacity, b.conic, b.geo, b.vaabb, b.vpair_offset, b.vprec, b.vwin,
                              b.gid_sorted, b.tile_offsets, rec, pat)
        ctx.meta = (b.n, b.h, b.w, b.overlap, b.total_pairs)
        return image

    @staticmethod
    def backward(ctx, grad_out):
        (scale, rot, feat, opacity, conic, geo, vaabb, vpair_offset, vprec, vwin, gid_sorted, tile_offsets, rec,
         pat) = ctx.saved_tensors
        n, h, w, overlap, total_pairs = ctx.meta
        b = FeatherBinned(n, h, w, overlap, conic, geo, vaabb, vpair_offset, vprec, vwin, total_pairs, gid_sorted,
                          tile_offsets)
        grad = grad_out.contiguous().float()
        with torch.cuda.device(scale.device):
            d_xy, _d_conic, d_feat, d_opacity, d_scale, d_rot = backward(b, aligned(feat, 4), opacity, scale, rot,
                                                                         grad, rec, pat)
        return d_xy, d_scale, d_rot, d_feat, d_opacity, None, None, None, None, None
