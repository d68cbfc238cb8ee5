"""Host orchestration of the render pipeline over the C ABI.

prepare -> (one 8-byte device->host read of the pair total) -> bin -> forward;
backward reuses the binning of its forward.  PyTorch only provides device
memory, the current stream and autograd plumbing; every kernel is in
liboss_b200.so.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from . import _lib

INT32_MAX = 2**31 - 1


def binning_mode(binning: str | None, default: str | None = None) -> int:
    """Map a binning name to its C-ABI code.

    Default ("exact56") reproduces the reference op's full-tail sum to within
    e^-28 = 6.9e-13 per unit of feature of every Gaussian it leaves out at a
    pixel ("exact", q = 176 lists, leaves out only weights below the smallest
    normal fp32); the environment variable OSS_RASTER_BINNING overrides the
    default.
    """
    name = binning if binning is not None else os.environ.get("OSS_RASTER_BINNING", default or _lib.DEFAULT_BINNING)
    name = name.strip().lower()
    if name not in _lib.BINNING_MODES:
        raise ValueError(f"binning must be one of {sorted(_lib.BINNING_MODES)}; got {name!r}")
    return _lib.BINNING_MODES[name]


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def check_float_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be CUDA")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be fp32")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def check_int_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be CUDA")
    if t.dtype != torch.int32:
        raise RuntimeError(f"{name} must be int32")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def aligned(t: torch.Tensor, nbytes: int) -> torch.Tensor:
    """Return t, or an aligned copy if its data pointer is not nbytes-aligned."""
    if t.numel() > 0 and t.data_ptr() % nbytes != 0:
        return t.clone()
    return t


def check_gaussians(xy, scale, rot, feat=None) -> tuple[int, int]:
    check_float_cuda(xy, "xy")
    check_float_cuda(scale, "scale")
    check_float_cuda(rot, "rot")
    if xy.dim() != 2 or xy.size(1) != 2:
        raise RuntimeError("xy must be (N,2)")
    if scale.dim() != 2 or scale.size(1) != 2:
        raise RuntimeError("scale must be (N,2)")
    if rot.dim() != 1:
        raise RuntimeError("rot must be (N,)")
    if xy.size(0) != scale.size(0):
        raise RuntimeError("xy/scale N mismatch")
    if xy.size(0) != rot.size(0):
        raise RuntimeError("xy/rot N mismatch")
    f = 0
    if feat is not None:
        check_float_cuda(feat, "feat")
        if feat.dim() != 2:
            raise RuntimeError("feat must be (N,F)")
        if xy.size(0) != feat.size(0):
            raise RuntimeError("xy/feat N mismatch")
        f = int(feat.size(1))
        if f > _lib.MAX_CHANNELS:
            raise RuntimeError("F must be <= 64")
    n = int(xy.size(0))
    if n > INT32_MAX:
        raise RuntimeError("N exceeds int32 range")
    return n, f


def check_hw(h: int, w: int, tile_size: int) -> tuple[int, int, int, int]:
    if h < 0 or w < 0:
        raise RuntimeError("H and W must be non-negative")
    if tile_size != _lib.TILE:
        raise RuntimeError("tile_size must be 16")
    if h > INT32_MAX:
        raise RuntimeError("H exceeds int32 range")
    if w > INT32_MAX:
        raise RuntimeError("W exceeds int32 range")
    ntx = (w + _lib.TILE - 1) // _lib.TILE
    nty = (h + _lib.TILE - 1) // _lib.TILE
    if ntx * nty > INT32_MAX:
        raise RuntimeError("number of tiles exceeds int32 range")
    return ntx, nty, ntx * nty, 0


@dataclass
class Binned:
    """Per-Gaussian records and per-tile lists of one render."""

    n: int
    h: int
    w: int
    mode: int
    conic: torch.Tensor        # (N, 3)
    aabb: torch.Tensor         # (N, 4) int32
    pair_offset: torch.Tensor  # (N+1,) int32, gid-major pair offsets
    geo: torch.Tensor          # (N, 8) raster records
    total_pairs: int
    gid_sorted: torch.Tensor   # (P,) int32
    tile_offsets: torch.Tensor  # (T+1,) int32
    prec: torch.Tensor | None = None  # (N, entry_record_floats(prec_f)) packed forward records
    prec_f: int = -1


_HOST_TOTAL = {}


def read_total(total: torch.Tensor, stream: int) -> int:
    """The device pair total on the host: a one-thread kernel stores it into
    mapped pinned memory and the host waits on an event -- the path's one host
    synchronisation, which so does not queue behind large copies in flight."""
    key = (total.device.index, stream)
    slot = _HOST_TOTAL.get(key)
    if slot is None:
        slot = (torch.empty((1,), dtype=torch.int64).pin_memory(), torch.cuda.Event())
        _HOST_TOTAL[key] = slot
    host, ev = slot
    _lib.check(_lib.lib().oss_publish_total(total.data_ptr(), host.data_ptr(), stream), "oss_publish_total")
    ev.record(torch.cuda.current_stream(total.device))
    ev.synchronize()
    return int(host[0])


def depth_order(depth: torch.Tensor):
    """(order, rank) of the Gaussians sorted by (depth, gid): the alpha-blend list key."""
    lib = _lib.lib()
    n = int(depth.numel())
    dev = depth.device
    order = torch.empty((n,), device=dev, dtype=torch.int32)
    rank = torch.empty((n,), device=dev, dtype=torch.int32)
    scratch = torch.empty((max(1, lib.oss_depth_order_scratch_bytes(n)),), device=dev, dtype=torch.uint8)
    _lib.check(lib.oss_depth_order(n, depth.data_ptr(), order.data_ptr(), rank.data_ptr(), scratch.data_ptr(),
                                   scratch.numel(), stream_of(depth)), "oss_depth_order")
    return order, rank


_STICKY_OVERFLOW = {}


def sticky_overflow(device) -> torch.Tensor:
    """Per-device int32 flag that capacity-mode binning ORs its overflow into."""
    idx = torch.device(device).index
    flag = _STICKY_OVERFLOW.get(idx)
    if flag is None:
        flag = torch.zeros((1,), device=torch.device("cuda", idx), dtype=torch.int32)
        _STICKY_OVERFLOW[idx] = flag
    return flag


def pair_capacity_overflowed(device=None, reset: bool = True) -> bool:
    """True if a capacity-mode call on `device` since the last check had more
    pairs than its capacity (its lists were emptied: zero image and gradients).
    A host synchronisation with the device."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flag = sticky_overflow(dev)
    hit = bool(int(flag.item()))
    if reset:
        flag.zero_()
    return hit


def bin_gaussians(xy: torch.Tensor, scale: torch.Tensor, rot: torch.Tensor, h: int, w: int, mode: int,
                  depth: torch.Tensor | None = None, capacity: int | None = None, feat: torch.Tensor | None = None,
                  opacity: torch.Tensor | None = None) -> Binned:
    """Preprocess + deterministic tile binning.  One host sync (the pair total)
    except in full mode, where the total N*T is known up front, and in capacity
    mode, where the lists are sized for `capacity` pairs, the device checks the
    total and raises the sticky overflow flag instead (no host sync).  With depth
    the tile lists are ordered by (depth, gid) instead of gid (alpha blending).
    With feat (and optionally opacity) the preprocess also packs the forward
    records of the additive render (one gathered line per list entry)."""
    lib = _lib.lib()
    n = int(xy.size(0))
    _, _, num_tiles, _ = check_hw(h, w, _lib.TILE)
    if mode == _lib.OSS_BIN_FULL and n > 0 and num_tiles > INT32_MAX // n:
        raise RuntimeError("full-frame raster pair count exceeds int32 range")
    dev = xy.device
    xy = aligned(xy, 8)
    scale = aligned(scale, 8)
    stream = stream_of(xy)
    f32 = dict(device=dev, dtype=torch.float32)
    i32 = dict(device=dev, dtype=torch.int32)
    conic = torch.empty((n, 3), **f32)
    aabb = torch.empty((n, 4), **i32)
    pair_offset = torch.empty((n + 1,), **i32)
    geo = torch.empty((n, 8), **f32)
    prec, prec_f = None, -1
    if feat is not None:
        prec_f = int(feat.size(1))
        feat = aligned(feat, 4)
        prec = torch.empty((n, lib.oss_entry_record_floats(prec_f)), **f32)
    total = torch.empty((1,), device=dev, dtype=torch.int64)
    tile_count = torch.empty((max(1, lib.oss_tile_count_elems(num_tiles)),), **i32)
    tile_offsets = torch.empty((num_tiles + 1,), **i32)
    if capacity is not None and depth is None and mode != _lib.OSS_BIN_FULL:
        # known capacity: preprocess, offsets and sorted lists in one call (three launches)
        capacity = int(capacity)
        if capacity > INT32_MAX:
            raise RuntimeError("total pair count exceeds int32 range")
        gid_sorted = torch.empty((capacity,), **i32)
        overflow = torch.empty((1,), **i32)
        scratch = torch.empty((max(1, lib.oss_render_bin_scratch_bytes(n, capacity, num_tiles)),), device=dev,
                              dtype=torch.uint8)
        _lib.check(
            lib.oss_render_bin(n, h, w, 1, None, mode, xy.data_ptr(), scale.data_ptr(), rot.data_ptr(),
                               max(prec_f, 0),
                               _lib.ptr(feat), _lib.ptr(opacity if feat is not None else None), conic.data_ptr(),
                               aabb.data_ptr(), pair_offset.data_ptr(), geo.data_ptr(), _lib.ptr(prec),
                               total.data_ptr(), tile_count.data_ptr(), tile_offsets.data_ptr(), capacity,
                               gid_sorted.data_ptr(), overflow.data_ptr(), scratch.data_ptr(), scratch.numel(),
                               stream),
            "oss_render_bin",
        )
        sticky_overflow(dev).bitwise_or_(overflow)
        return Binned(n, h, w, mode, conic, aabb, pair_offset, geo, capacity, gid_sorted, tile_offsets, prec, prec_f)
    scratch = torch.empty((max(1, lib.oss_render_prepare_scratch_bytes(n)),), device=dev, dtype=torch.uint8)
    _lib.check(
        lib.oss_render_prepare(n, h, w, mode, xy.data_ptr(), scale.data_ptr(), rot.data_ptr(), max(prec_f, 0),
                               _lib.ptr(feat), _lib.ptr(opacity if feat is not None else None), conic.data_ptr(),
                               aabb.data_ptr(), pair_offset.data_ptr(), geo.data_ptr(), _lib.ptr(prec),
                               total.data_ptr(), tile_count.data_ptr(), tile_offsets.data_ptr(), scratch.data_ptr(),
                               scratch.numel(), stream),
        "oss_render_prepare",
    )
    if mode == _lib.OSS_BIN_FULL:
        total_pairs = n * num_tiles
    elif capacity is not None:
        total_pairs = int(capacity)
    else:
        total_pairs = read_total(total, stream)
    if total_pairs > INT32_MAX:
        raise RuntimeError("total pair count exceeds int32 range")
    gid_sorted = torch.empty((total_pairs,), **i32)
    overflow = torch.empty((1,), **i32)
    nbytes = lib.oss_bin_pairs_scratch_bytes(n, total_pairs, num_tiles)
    scratch2 = torch.empty((max(1, nbytes),), device=dev, dtype=torch.uint8)
    order = rank = None
    if depth is not None and mode != _lib.OSS_BIN_FULL:
        order, rank = depth_order(depth)
    # without a capacity, total_pairs is the exact total read above and the check cannot fire
    _lib.check(
        lib.oss_bin_pairs(n, h, w, mode, aabb.data_ptr(), pair_offset.data_ptr(), tile_count.data_ptr(),
                          total.data_ptr(), total_pairs, _lib.ptr(rank), _lib.ptr(order), gid_sorted.data_ptr(),
                          tile_offsets.data_ptr(), overflow.data_ptr(), scratch2.data_ptr(), scratch2.numel(),
                          stream),
        "oss_bin_pairs",
    )
    if capacity is not None and mode != _lib.OSS_BIN_FULL:
        sticky_overflow(dev).bitwise_or_(overflow)
    return Binned(n, h, w, mode, conic, aabb, pair_offset, geo, total_pairs, gid_sorted, tile_offsets, prec, prec_f)


def render_forward(b: Binned, feat: torch.Tensor, opacity: torch.Tensor | None, records: bool = False):
    """(F, H, W) image; with records=True also the per-entry records the
    backward reads (returns (image, records, slots); slots is None: the backward
    derives the pair slots from the lists).  Uses the packed records of
    bin_gaussians(feat=...) when they were made for these features."""
    lib = _lib.lib()
    f = int(feat.size(1))
    dev = feat.device
    image = torch.empty((f, b.h, b.w), device=dev, dtype=torch.float32)
    rec = slots = None
    if records and b.mode != _lib.OSS_BIN_FULL and b.total_pairs > 0:
        rec = torch.empty((b.total_pairs, lib.oss_entry_record_floats(f)), device=dev, dtype=torch.float32)
    prec = b.prec if b.prec is not None and b.prec_f == f else None
    _lib.check(
        lib.oss_render_forward(b.n, f, b.h, b.w, b.geo.data_ptr(), feat.data_ptr(), _lib.ptr(opacity),
                               _lib.ptr(prec), b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(),
                               image.data_ptr(), b.aabb.data_ptr(), b.pair_offset.data_ptr(), _lib.ptr(rec),
                               _lib.ptr(slots), stream_of(feat)),
        "oss_render_forward",
    )
    if records:
        return image, rec, slots
    return image


def render_backward(b: Binned, feat: torch.Tensor, opacity: torch.Tensor | None, scale: torch.Tensor,
                    rot: torch.Tensor, grad_image: torch.Tensor, records: torch.Tensor | None = None,
                    slots: torch.Tensor | None = None):
    """Deterministic gradients (d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot);
    records/slots are the forward's entry records (None: gathered again)."""
    lib = _lib.lib()
    dev = feat.device
    n, f = b.n, int(feat.size(1))
    f32 = dict(device=dev, dtype=torch.float32)
    d_xy = torch.empty((n, 2), **f32)
    d_conic = torch.empty((n, 3), **f32)
    d_feat = torch.empty((n, f), **f32)
    d_opacity = torch.empty((n,), **f32) if opacity is not None else None
    d_scale = torch.empty((n, 2), **f32)
    d_rot = torch.empty((n,), **f32)
    num_tiles = int(b.tile_offsets.numel()) - 1
    nbytes = lib.oss_render_backward_scratch_bytes(b.total_pairs, f, num_tiles)
    scratch = torch.empty((max(1, nbytes),), device=dev, dtype=torch.uint8)
    scale = aligned(scale, 8)
    _lib.check(
        lib.oss_render_backward(n, f, b.h, b.w, b.geo.data_ptr(), feat.data_ptr(), _lib.ptr(opacity),
                                scale.data_ptr(), rot.data_ptr(), b.aabb.data_ptr(), b.pair_offset.data_ptr(),
                                b.total_pairs, b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(), _lib.ptr(records),
                                _lib.ptr(slots), grad_image.data_ptr(), d_xy.data_ptr(), d_conic.data_ptr(),
                                d_feat.data_ptr(),
                                _lib.ptr(d_opacity), d_scale.data_ptr(), d_rot.data_ptr(), scratch.data_ptr(),
                                scratch.numel(), stream_of(feat)),
        "oss_render_backward",
    )
    return d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot


def render_analytic_forward(b: Binned, feat: torch.Tensor, opacity: torch.Tensor | None) -> torch.Tensor:
    """(F, H, W) with the Analytic-Splatting pixel integral as the weight (F <= 32)."""
    lib = _lib.lib()
    f = int(feat.size(1))
    image = torch.empty((f, b.h, b.w), device=feat.device, dtype=torch.float32)
    _lib.check(lib.oss_render_analytic_forward(b.n, f, b.h, b.w, b.geo.data_ptr(), feat.data_ptr(), _lib.ptr(opacity),
                                               b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(), image.data_ptr(),
                                               stream_of(feat)), "oss_render_analytic_forward")
    return image


def render_analytic_backward(b: Binned, feat: torch.Tensor, opacity: torch.Tensor | None, scale: torch.Tensor,
                             rot: torch.Tensor, grad_image: torch.Tensor):
    """(d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot) of the analytic-weight render."""
    lib = _lib.lib()
    dev = feat.device
    n, f = b.n, int(feat.size(1))
    f32 = dict(device=dev, dtype=torch.float32)
    d_xy, d_conic, d_feat = torch.empty((n, 2), **f32), torch.empty((n, 3), **f32), torch.empty((n, f), **f32)
    d_opacity = torch.empty((n,), **f32) if opacity is not None else None
    d_scale, d_rot = torch.empty((n, 2), **f32), torch.empty((n,), **f32)
    nbytes = lib.oss_render_analytic_backward_scratch_bytes(b.total_pairs, f)
    scratch = torch.empty((max(1, nbytes),), device=dev, dtype=torch.uint8)
    scale = aligned(scale, 8)
    _lib.check(lib.oss_render_analytic_backward(n, f, b.h, b.w, b.geo.data_ptr(), feat.data_ptr(), _lib.ptr(opacity),
                                                scale.data_ptr(), rot.data_ptr(), b.aabb.data_ptr(),
                                                b.pair_offset.data_ptr(), b.total_pairs, b.gid_sorted.data_ptr(),
                                                b.tile_offsets.data_ptr(), grad_image.data_ptr(), d_xy.data_ptr(),
                                                d_conic.data_ptr(), d_feat.data_ptr(), _lib.ptr(d_opacity),
                                                d_scale.data_ptr(), d_rot.data_ptr(), scratch.data_ptr(),
                                                scratch.numel(), stream_of(feat)), "oss_render_analytic_backward")
    return d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot


def background_vector(background, f: int, device) -> torch.Tensor | None:
    """None, a scalar or F values -> a device (F,) fp32 tensor (None stays None)."""
    if background is None:
        return None
    bg = torch.as_tensor(background, dtype=torch.float32, device=device).reshape(-1)
    if bg.numel() == 1:
        bg = bg.expand(f)
    if bg.numel() != f:
        raise RuntimeError("background must be a scalar or have F values")
    return bg.contiguous()


def render_alpha_forward(b: Binned, feat: torch.Tensor, opacity: torch.Tensor | None,
                         background: torch.Tensor | None):
    """(image (F,H,W), t_final (H,W), n_contrib (H,W) int32) of front-to-back compositing."""
    lib = _lib.lib()
    f = int(feat.size(1))
    dev = feat.device
    image = torch.empty((f, b.h, b.w), device=dev, dtype=torch.float32)
    t_final = torch.empty((b.h, b.w), device=dev, dtype=torch.float32)
    n_contrib = torch.empty((b.h, b.w), device=dev, dtype=torch.int32)
    _lib.check(
        lib.oss_render_alpha_forward(b.n, f, b.h, b.w, b.geo.data_ptr(), feat.data_ptr(), _lib.ptr(opacity),
                                     _lib.ptr(background), b.gid_sorted.data_ptr(), b.tile_offsets.data_ptr(),
                                     image.data_ptr(), t_final.data_ptr(), n_contrib.data_ptr(), stream_of(feat)),
        "oss_render_alpha_forward",
    )
    return image, t_final, n_contrib


def render_alpha_backward(b: Binned, feat: torch.Tensor, opacity: torch.Tensor | None,
                          background: torch.Tensor | None, scale: torch.Tensor, rot: torch.Tensor,
                          t_final: torch.Tensor, n_contrib: torch.Tensor, grad_image: torch.Tensor):
    """Deterministic (d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot) of the alpha blend."""
    lib = _lib.lib()
    dev = feat.device
    n, f = b.n, int(feat.size(1))
    f32 = dict(device=dev, dtype=torch.float32)
    d_xy = torch.empty((n, 2), **f32)
    d_conic = torch.empty((n, 3), **f32)
    d_feat = torch.empty((n, f), **f32)
    d_opacity = torch.empty((n,), **f32)
    d_scale = torch.empty((n, 2), **f32)
    d_rot = torch.empty((n,), **f32)
    nbytes = lib.oss_render_alpha_backward_scratch_bytes(b.total_pairs, f)
    scratch = torch.empty((max(16, nbytes),), device=dev, dtype=torch.uint8)
    scale = aligned(scale, 8)
    _lib.check(
        lib.oss_render_alpha_backward(n, f, b.h, b.w, b.geo.data_ptr(), feat.data_ptr(), _lib.ptr(opacity),
                                      _lib.ptr(background), scale.data_ptr(), rot.data_ptr(), b.aabb.data_ptr(),
                                      b.pair_offset.data_ptr(), b.total_pairs, b.gid_sorted.data_ptr(),
                                      b.tile_offsets.data_ptr(), t_final.data_ptr(), n_contrib.data_ptr(),
                                      grad_image.data_ptr(), d_xy.data_ptr(), d_conic.data_ptr(), d_feat.data_ptr(),
                                      d_opacity.data_ptr(), d_scale.data_ptr(), d_rot.data_ptr(), scratch.data_ptr(),
                                      scratch.numel(), stream_of(feat)),
        "oss_render_alpha_backward",
    )
    return d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot
