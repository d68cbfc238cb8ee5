"""B frames in one launch chain (rasterize_gaussians_batched).

Frame b is drawn from Gaussians [offsets[b], offsets[b+1]) of the concatenated
inputs.  The C ABI bins all frames at once on a grid of the frames' tiles
stacked (oss_render_bin with frames = B): each frame's lists are the ones a
call on its Gaussians alone builds, so the images and gradients are those of
B separate calls, bit for bit, from one preprocess, one scatter, one forward,
one backward and one reduce instead of B of each.  The reference renders a
batch by calling its op once per frame (oss/sr/v6/model.py:795-820).
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from . import _lib
from ._raster import INT32_MAX, aligned, read_total, stream_of, sticky_overflow


_FRAME_OFFSETS = {}  # (device, offsets) -> device tensor, least recently used first
_CAPTURED = set()  # keys used inside a CUDA-graph capture: the graph reads them on every replay
_MAX_UNCAPTURED = 64


def frame_offsets_on(device, offsets) -> torch.Tensor:
    """The frame offsets as a device int32 tensor, made once per device and
    offsets (a host copy would break CUDA-graph capture of later calls).

    A tensor used while a graph was being captured is kept for the life of the
    process, since the graph keeps its address; of the others, the least
    recently used is dropped beyond 64 (kernels already queued that read it
    keep its memory: the tensor is recorded on each stream that used it)."""
    dev = torch.device(device)
    key = (dev.index, tuple(int(v) for v in offsets))
    t = _FRAME_OFFSETS.pop(key, None)
    if t is None:
        t = torch.tensor(key[1], device=dev, dtype=torch.int32)
    _FRAME_OFFSETS[key] = t
    if torch.cuda.is_current_stream_capturing():
        _CAPTURED.add(key)
    else:
        t.record_stream(torch.cuda.current_stream(dev))
        spare = [k for k in _FRAME_OFFSETS if k not in _CAPTURED]
        for k in spare[:max(0, len(spare) - _MAX_UNCAPTURED)]:
            del _FRAME_OFFSETS[k]
    return t


class BinnedFrames:
    """Lists and per-Gaussian records of one batched binning."""

    def __init__(self, n, frames, h, w, mode, conic, aabb, pair_offset, geo, prec, prec_f, total_pairs, gid_sorted,
                 tile_offsets):
        self.n, self.frames, self.h, self.w, self.mode = n, frames, h, w, mode
        self.conic, self.aabb, self.pair_offset, self.geo = conic, aabb, pair_offset, geo
        self.prec, self.prec_f = prec, prec_f
        self.total_pairs, self.gid_sorted, self.tile_offsets = total_pairs, gid_sorted, tile_offsets

    @property
    def num_tiles(self) -> int:
        return int(self.tile_offsets.numel()) - 1


def bin_frames(xy, scale, rot, h, w, mode, offsets, feat, opacity, capacity=None) -> BinnedFrames:
    """Preprocess + lists of every frame in one call.  Without a capacity the
    pair total is measured first (one call that only counts, then a host read),
    with one the device checks it and raises the sticky overflow flag."""
    lib = _lib.lib()
    n = int(xy.size(0))
    frames = len(offsets) - 1
    dev = xy.device
    ntx, nty = (w + _lib.TILE - 1) // _lib.TILE, (h + _lib.TILE - 1) // _lib.TILE
    tiles = ntx * nty * frames
    xy, scale = aligned(xy, 8), aligned(scale, 8)
    feat = aligned(feat, 4)
    stream = stream_of(xy)
    f32 = dict(device=dev, dtype=torch.float32)
    i32 = dict(device=dev, dtype=torch.int32)
    f = int(feat.size(1))
    fo = frame_offsets_on(dev, offsets)
    conic = torch.empty((n, 3), **f32)
    aabb = torch.empty((n, 4), **i32)
    pair_offset = torch.empty((n + 1,), **i32)
    geo = torch.empty((n, 8), **f32)
    prec = torch.empty((n, lib.oss_entry_record_floats(f)), **f32)
    total = torch.empty((1,), device=dev, dtype=torch.int64)
    tile_count = torch.empty((max(1, lib.oss_tile_count_elems(tiles)),), **i32)
    tile_offsets = torch.empty((tiles + 1,), **i32)
    overflow = torch.empty((1,), **i32)

    def run(cap, gid_sorted):
        scratch = torch.empty((max(1, lib.oss_render_bin_scratch_bytes(n, cap, tiles)),), device=dev,
                              dtype=torch.uint8)
        _lib.check(
            lib.oss_render_bin(n, h, w, frames, fo.data_ptr(), mode, xy.data_ptr(), scale.data_ptr(), rot.data_ptr(),
                               f, feat.data_ptr(), _lib.ptr(opacity), conic.data_ptr(), aabb.data_ptr(),
                               pair_offset.data_ptr(), geo.data_ptr(), prec.data_ptr(), total.data_ptr(),
                               tile_count.data_ptr(), tile_offsets.data_ptr(), cap, gid_sorted.data_ptr(),
                               overflow.data_ptr(), scratch.data_ptr(), scratch.numel(), stream),
            "oss_render_bin",
        )

    if capacity is None:
        run(0, torch.empty((1,), **i32))  # counts only: the lists overflow and come out empty
        capacity = read_total(total, stream)
        if capacity > INT32_MAX:
            raise RuntimeError("total pair count exceeds int32 range")
        gid_sorted = torch.empty((max(1, capacity),), **i32)
        run(capacity, gid_sorted)
    else:
        gid_sorted = torch.empty((max(1, capacity),), **i32)
        run(capacity, gid_sorted)
        sticky_overflow(dev).bitwise_or_(overflow)
    return BinnedFrames(n, frames, h, w, mode, conic, aabb, pair_offset, geo, prec, f, capacity, gid_sorted,
                        tile_offsets)


def forward_frames(b: BinnedFrames, feat, records: bool):
    """([B, F, H, W] image, entry records or None)."""
    lib = _lib.lib()
    f = int(feat.size(1))
    image = torch.empty((b.frames, f, b.h, b.w), device=feat.device, dtype=torch.float32)
    rec = None
    if records and b.total_pairs > 0:
        rec = torch.empty((b.total_pairs, lib.oss_entry_record_floats(f)), device=feat.device, dtype=torch.float32)
    _lib.check(
        lib.oss_render_forward_frames(b.n, f, b.h, b.w, b.frames, None, None, None, b.prec.data_ptr(),
                                      b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(), image.data_ptr(), None,
                                      None, _lib.ptr(rec), None, stream_of(feat)),
        "oss_render_forward_frames",
    )
    return image, rec


def backward_frames(b: BinnedFrames, feat, opacity, scale, rot, grad, records):
    """(d_xy, d_feat, d_opacity, d_scale, d_rot): the table-driven backward over
    every frame's tiles, then the per-Gaussian reduce."""
    lib = _lib.lib()
    dev = feat.device
    n, f = b.n, int(feat.size(1))
    stream = stream_of(feat)
    f32 = dict(device=dev, dtype=torch.float32)
    stride = lib.oss_pair_grad_stride(f)
    pg = torch.empty((max(1, b.total_pairs) * stride,), **f32)
    nbytes = lib.oss_render_backward_pairs_scratch_bytes(b.total_pairs, b.num_tiles)
    items = torch.empty((max(1, nbytes),), device=dev, dtype=torch.uint8)
    _lib.check(lib.oss_backward_items_frames(b.h, b.w, b.frames, b.total_pairs, b.tile_offsets.data_ptr(),
                                             items.data_ptr(), items.numel(), stream), "oss_backward_items_frames")
    _lib.check(
        lib.oss_render_backward_items_frames(n, f, b.h, b.w, b.frames, b.geo.data_ptr(), feat.data_ptr(),
                                             _lib.ptr(opacity), b.aabb.data_ptr(), b.pair_offset.data_ptr(),
                                             b.total_pairs, b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(),
                                             _lib.ptr(records), None, grad.data_ptr(), pg.data_ptr(),
                                             items.data_ptr(), items.numel(), stream),
        "oss_render_backward_items_frames",
    )
    d_xy = torch.empty((n, 2), **f32)
    d_conic = torch.empty((n, 3), **f32)
    d_feat = torch.empty((n, f), **f32)
    d_opacity = torch.empty((n,), **f32) if opacity is not None else None
    d_scale = torch.empty((n, 2), **f32)
    d_rot = torch.empty((n,), **f32)
    _lib.check(
        lib.oss_reduce_pair_grads(n, f, pg.data_ptr(), b.pair_offset.data_ptr(), b.geo.data_ptr(), feat.data_ptr(),
                                  _lib.ptr(opacity), aligned(scale, 8).data_ptr(), rot.data_ptr(), d_xy.data_ptr(),
                                  d_conic.data_ptr(), d_feat.data_ptr(), _lib.ptr(d_opacity), d_scale.data_ptr(),
                                  d_rot.data_ptr(), stream),
        "oss_reduce_pair_grads",
    )
    return d_xy, d_feat, d_opacity, d_scale, d_rot


class RasterizeFrames(Function):
    """(B, F, H, W) from B frames of concatenated Gaussians, one launch chain."""

    @staticmethod
    def forward(ctx, xy, scale, rot, feat, opacity, offsets, h, w, mode, capacity):
        with torch.cuda.device(xy.device):
            b = bin_frames(xy, scale, rot, h, w, mode, offsets, feat, opacity, capacity)
            image, records = forward_frames(b, feat, any(ctx.needs_input_grad[:5]))
        # the backward reads the forward's entry records, not the packed per-Gaussian ones
        ctx.save_for_backward(xy, scale, rot, feat, opacity, b.conic, b.aabb, b.pair_offset, b.geo, b.gid_sorted,
                              b.tile_offsets, records)
        ctx.meta = (b.n, b.frames, h, w, mode, b.total_pairs, b.prec_f)
        return image

    @staticmethod
    def backward(ctx, grad_out):
        (xy, scale, rot, feat, opacity, conic, aabb, pair_offset, geo, gid_sorted, tile_offsets,
         records) = ctx.saved_tensors
        n, frames, h, w, mode, total_pairs, prec_f = ctx.meta
        b = BinnedFrames(n, frames, h, w, mode, conic, aabb, pair_offset, geo, None, prec_f, total_pairs, gid_sorted,
                         tile_offsets)
        grad = grad_out.contiguous()
        if grad.dtype != torch.float32:
            grad = grad.float()
        with torch.cuda.device(xy.device):
            d_xy, d_feat, d_opacity, d_scale, d_rot = backward_frames(b, aligned(feat, 4), opacity, scale, rot, grad,
                                                                      records)
        return d_xy, d_scale, d_rot, d_feat, d_opacity, None, None, None, None, None
