"""numpy front-end of the CPU oracle (oracle/oss_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker; never by the product package.

    python oracle/oracle.py --build      # compile liboss_oracle.so with gcc
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "oss_oracle.c"
LIB = ORACLE_DIR / "liboss_oracle.so"

TIGHT, EXACT, FULL = 0, 1, 2
MODES = {"tight3sigma": TIGHT, "exact": EXACT, "full": FULL}
TILE = 16

CFLAGS = ["-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-msse2",
          "-mfpmath=sse"]


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = ["gcc", *CFLAGS, str(SRC), "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB))
        i64, i32, p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        _lib.orc_preprocess.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p]
        _lib.orc_pair_construction.argtypes = [i64, i32, i32, p, p, p, p]
        _lib.orc_pair_construction.restype = i64
        _lib.orc_full_pairs.argtypes = [i64, i64, p, p]
        _lib.orc_render_forward.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p, p, i64, i64]
        _lib.orc_render_backward.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p, p, p, p, p, p, i64, i64]
        _lib.orc_conic_to_scale_rot_grad.argtypes = [i64, p, p, p, p, p]
        _lib.orc_render_alpha_forward.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p, p, p, p, p, p, i64, i64]
        _lib.orc_render_alpha_backward.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p, p, p, p, p, p, p, i64, i64]
        _lib.orc_tile_bin_counting_sort.argtypes = [i64, i64, p, p, p, p]
        _lib.orc_num_threads.restype = i32
        _lib.orc_set_num_threads.argtypes = [i32]
        f32 = ctypes.c_float
        _lib.orc_warp_canvas.argtypes = [i64, i32, i32, i32, i32, i32, p, f32, p, p, p, p, p, p, p, p, p, p, p]
        _lib.orc_warp_canvas.restype = i64
        _lib.orc_warp_positions.argtypes = [i64, i32, i32, p, f32, p, p, p]
    return _lib


def warp_canvas(positions, scales, rotations, opacities, colors, motion_lr, hw, sigma_recon=0.5, alpha=1.0):
    """GS-STVSR canvas warp (oss/sr/v6/canvas_warp.py:177-254) with motion
    pre-multiplied by alpha; returns the compacted canvas arrays and count."""
    pos, sc, rt, op, col = _f32(positions), _f32(scales), _f32(rotations), _f32(opacities), _f32(colors)
    m = _f32(motion_lr)
    if m.ndim == 4:
        m = np.ascontiguousarray(m[0])
    n, f = col.shape
    h, w = int(hw[0]), int(hw[1])
    rec = np.asarray(sigma_recon, np.float32)
    rec = _f32(np.eye(2, dtype=np.float32) * rec) if rec.ndim == 0 else _f32(rec.reshape(2, 2))
    outs = [np.empty((n, 2), np.float32), np.empty((n, 2), np.float32), np.empty((n,), np.float32),
            np.empty((n,), np.float32), np.empty((n, f), np.float32)]
    k = lib().orc_warp_canvas(n, f, m.shape[1], m.shape[2], h, w, _p(m), float(alpha), _p(rec), _p(pos), _p(sc),
                              _p(rt), _p(op), _p(col), *(_p(o) for o in outs))
    return tuple(o[:k] for o in outs) + (int(k),)


def warp_positions(xy, motion, hw, alpha=1.0):
    """oss/gaussian/canvas/warp.py:28-91 with motion * alpha; (new_xy, in_frame)."""
    xy, m = _f32(xy), _f32(motion)
    n = xy.shape[0]
    out = np.empty((n, 2), np.float32)
    flag = np.empty((n,), np.uint8)
    lib().orc_warp_positions(n, int(hw[0]), int(hw[1]), _p(m), float(alpha), _p(xy), _p(out), _p(flag))
    return out, flag.astype(bool)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def tiles(h: int, w: int) -> tuple[int, int, int]:
    ntx = (w + TILE - 1) // TILE
    nty = (h + TILE - 1) // TILE
    return ntx, nty, ntx * nty


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(t: int) -> None:
    lib().orc_set_num_threads(int(t))


def preprocess(xy, scale, rot, h, w, mode=TIGHT):
    """(conic (N,3), aabb (N,4) int32, count (N,) int32) -- rasterizer_fwd.cu:38-109."""
    xy, scale, rot = _f32(xy), _f32(scale), _f32(rot)
    n = xy.shape[0]
    conic = np.empty((n, 3), np.float32)
    aabb = np.empty((n, 4), np.int32)
    count = np.empty((n,), np.int32)
    lib().orc_preprocess(n, h, w, mode, _p(xy), _p(scale), _p(rot), _p(conic), _p(aabb), _p(count))
    return conic, aabb, count


def pair_construction(aabb, count, h, w):
    """(gid_sorted, tile_offsets) sorted by (tile << 32 | gid) -- rasterizer_fwd.cu:446-475."""
    aabb, count = _i32(aabb), _i32(count)
    total = int(count.astype(np.int64).sum())
    _, _, t = tiles(h, w)
    gid = np.empty((max(total, 1),), np.int32)
    offs = np.empty((t + 1,), np.int32)
    got = lib().orc_pair_construction(aabb.shape[0], h, w, _p(aabb), _p(count), _p(gid), _p(offs))
    assert got == total
    return gid[:total], offs


def full_pairs(n, h, w):
    _, _, t = tiles(h, w)
    gid = np.empty((max(n * t, 1),), np.int32)
    offs = np.empty((t + 1,), np.int32)
    lib().orc_full_pairs(n, t, _p(gid), _p(offs))
    return gid[: n * t], offs


def lists(xy, scale, rot, h, w, mode=TIGHT):
    """(conic, aabb, count, gid_sorted, tile_offsets) for a binning mode."""
    conic, aabb, count = preprocess(xy, scale, rot, h, w, mode)
    if mode == FULL:
        gid, offs = full_pairs(conic.shape[0], h, w)
    else:
        gid, offs = pair_construction(aabb, count, h, w)
    return conic, aabb, count, gid, offs


def render_forward(xy, conic, feat, gid, offs, h, w, opacity=None, tile_range=None):
    xy, conic, feat = _f32(xy), _f32(conic), _f32(feat)
    gid, offs = _i32(gid), _i32(offs)
    op = None if opacity is None else _f32(opacity)
    n, f = feat.shape
    _, _, t = tiles(h, w)
    lo, hi = (0, t) if tile_range is None else tile_range
    out = np.zeros((f, h, w), np.float32)
    lib().orc_render_forward(n, f, h, w, _p(xy), _p(conic), _p(feat), _p(op), _p(gid), _p(offs), _p(out), lo, hi)
    return out


def render_backward(xy, conic, feat, gid, offs, grad, h, w, opacity=None, tile_range=None):
    """(d_xy, d_conic, d_feat, d_opacity) -- rasterizer_bwd.cu:78-109, double sums."""
    xy, conic, feat, grad = _f32(xy), _f32(conic), _f32(feat), _f32(grad)
    gid, offs = _i32(gid), _i32(offs)
    op = None if opacity is None else _f32(opacity)
    n, f = feat.shape
    _, _, t = tiles(h, w)
    lo, hi = (0, t) if tile_range is None else tile_range
    d_xy = np.empty((n, 2), np.float32)
    d_conic = np.empty((n, 3), np.float32)
    d_feat = np.empty((n, f), np.float32)
    d_op = np.empty((n,), np.float32) if op is not None else None
    lib().orc_render_backward(n, f, h, w, _p(xy), _p(conic), _p(feat), _p(op), _p(gid), _p(offs), _p(grad),
                              _p(d_xy), _p(d_conic), _p(d_feat), _p(d_op), lo, hi)
    return d_xy, d_conic, d_feat, d_op


def conic_to_scale_rot_grad(scale, rot, d_conic):
    scale, rot, d_conic = _f32(scale), _f32(rot), _f32(d_conic)
    n = scale.shape[0]
    d_scale = np.empty((n, 2), np.float32)
    d_rot = np.empty((n,), np.float32)
    lib().orc_conic_to_scale_rot_grad(n, _p(scale), _p(rot), _p(d_conic), _p(d_scale), _p(d_rot))
    return d_scale, d_rot


def tile_bin_counting_sort(tile_id, gid, num_tiles):
    tile_id, gid = _i32(tile_id), _i32(gid)
    n = tile_id.shape[0]
    out = np.empty((max(n, 1),), np.int32)
    offs = np.empty((num_tiles + 1,), np.int32)
    lib().orc_tile_bin_counting_sort(n, num_tiles, _p(tile_id), _p(gid), _p(out), _p(offs))
    return out[:n], offs


def render(xy, scale, rot, feat, h, w, mode=TIGHT, opacity=None):
    """Forward image through the oracle's own preprocess and lists."""
    conic, _, _, gid, offs = lists(xy, scale, rot, h, w, mode)
    return render_forward(xy, conic, feat, gid, offs, h, w, opacity)


def render_grads(xy, scale, rot, feat, grad, h, w, mode=TIGHT, opacity=None):
    """(d_xy, d_scale, d_rot, d_feat, d_opacity, d_conic) through the oracle's own lists."""
    conic, _, _, gid, offs = lists(xy, scale, rot, h, w, mode)
    d_xy, d_conic, d_feat, d_op = render_backward(xy, conic, feat, gid, offs, grad, h, w, opacity)
    d_scale, d_rot = conic_to_scale_rot_grad(scale, rot, d_conic)
    return d_xy, d_scale, d_rot, d_feat, d_op, d_conic


def depth_order_lists(gid, offs, depth):
    """Re-sort every tile list by (depth, gid) ascending: the list order of the
    alpha-blend mode (depth -0.0 counts as +0.0)."""
    gid, offs = _i32(gid), _i32(offs)
    d = _f32(depth) + np.float32(0.0)
    out = gid.copy()
    for t in range(offs.size - 1):
        b, e = int(offs[t]), int(offs[t + 1])
        if e - b > 1:
            seg = gid[b:e]
            out[b:e] = seg[np.lexsort((seg, d[seg]))]
    return out


def render_alpha_forward(xy, conic, feat, opacity, gid, offs, h, w, background=None, tile_range=None):
    """(image (F,H,W), t_final (H,W), n_contrib (H,W) int32, ambiguous (H,W) bool) of
    front-to-back compositing over the given lists (see oss_oracle.c)."""
    xy, conic, feat, op = _f32(xy), _f32(conic), _f32(feat), _f32(opacity)
    gid, offs = _i32(gid), _i32(offs)
    bg = None if background is None else _f32(np.broadcast_to(np.asarray(background, np.float32), (feat.shape[1],)))
    n, f = feat.shape
    _, _, t = tiles(h, w)
    lo, hi = (0, t) if tile_range is None else tile_range
    out = np.zeros((f, h, w), np.float32)
    tf = np.ones((h, w), np.float32)
    nc = np.zeros((h, w), np.int32)
    amb = np.zeros((h, w), np.uint8)
    lib().orc_render_alpha_forward(n, f, h, w, _p(xy), _p(conic), _p(feat), _p(op), _p(bg), _p(gid), _p(offs),
                                   _p(out), _p(tf), _p(nc), _p(amb), lo, hi)
    return out, tf, nc, amb.astype(bool)


def render_alpha_backward(xy, conic, feat, opacity, gid, offs, grad, h, w, background=None, tile_range=None):
    """(d_xy, d_conic, d_feat, d_opacity) of render_alpha_forward, double sums."""
    xy, conic, feat, op, grad = _f32(xy), _f32(conic), _f32(feat), _f32(opacity), _f32(grad)
    gid, offs = _i32(gid), _i32(offs)
    bg = None if background is None else _f32(np.broadcast_to(np.asarray(background, np.float32), (feat.shape[1],)))
    n, f = feat.shape
    _, _, t = tiles(h, w)
    lo, hi = (0, t) if tile_range is None else tile_range
    d_xy = np.empty((n, 2), np.float32)
    d_conic = np.empty((n, 3), np.float32)
    d_feat = np.empty((n, f), np.float32)
    d_op = np.empty((n,), np.float32)
    lib().orc_render_alpha_backward(n, f, h, w, _p(xy), _p(conic), _p(feat), _p(op), _p(bg), _p(gid), _p(offs),
                                    _p(grad), _p(d_xy), _p(d_conic), _p(d_feat), _p(d_op), lo, hi)
    return d_xy, d_conic, d_feat, d_op


def alpha_lists(xy, scale, rot, depth, h, w, mode=TIGHT):
    """(conic, gid_sorted by (tile, depth, gid), tile_offsets)."""
    conic, _, _, gid, offs = lists(xy, scale, rot, h, w, mode)
    return conic, (gid if depth is None else depth_order_lists(gid, offs, depth)), offs


def render_alpha(xy, scale, rot, feat, opacity, h, w, depth=None, background=None, mode=TIGHT):
    conic, gid, offs = alpha_lists(xy, scale, rot, depth, h, w, mode)
    return render_alpha_forward(xy, conic, feat, opacity, gid, offs, h, w, background)


def render_alpha_grads(xy, scale, rot, feat, opacity, grad, h, w, depth=None, background=None, mode=TIGHT):
    """(d_xy, d_scale, d_rot, d_feat, d_opacity, d_conic) of the alpha-blend render."""
    conic, gid, offs = alpha_lists(xy, scale, rot, depth, h, w, mode)
    d_xy, d_conic, d_feat, d_op = render_alpha_backward(xy, conic, feat, opacity, gid, offs, grad, h, w, background)
    d_scale, d_rot = conic_to_scale_rot_grad(scale, rot, d_conic)
    return d_xy, d_scale, d_rot, d_feat, d_op, d_conic


if __name__ == "__main__":
    if "--build" in sys.argv:
        print(build(force=True))
