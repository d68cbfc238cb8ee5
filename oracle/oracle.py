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

TIGHT, EXACT, FULL, EXACT56 = 0, 1, 2, 3
MODES = {"tight3sigma": TIGHT, "exact": EXACT, "full": FULL, "exact56": EXACT56}
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
        _lib.orc_render_backward_f32.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p, p, p, p, p, p, i64, i64, i32]
        _lib.orc_render_backward_exact.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p, p, p, p, p, p, i64, i64]
        _lib.orc_render_backward_fma.argtypes = [i64, i32, i32, i32, p, p, p, p, p, p, p, p, p, p, p, i64, i64]
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


def render_backward(xy, conic, feat, gid, offs, grad, h, w, opacity=None, tile_range=None, sums="f64"):
    """(d_xy, d_conic, d_feat, d_opacity) -- rasterizer_bwd.cu:78-109, double sums.
    sums="f32" / "f32r" sum in fp32 one pixel term at a time, as the reference's
    atomics do, in one order they may run in or in its reverse (the fp32
    evaluations the parity bar is judged beside); sums="exact" evaluates every
    per-pixel quantity in double too (the exact value at the fp32 inputs), and
    sums="f64fma" sums the terms whose q is formed with fused multiply-adds (as
    the reference's CUDA build contracts it)."""
    xy, conic, feat, grad = _f32(xy), _f32(conic), _f32(feat), _f32(grad)
    gid, offs = _i32(gid), _i32(offs)
    op = None if opacity is None else _f32(opacity)
    n, f = feat.shape
    _, _, t = tiles(h, w)
    lo, hi = (0, t) if tile_range is None else tile_range
    dt = np.float64 if sums == "exact" else np.float32  # the exact value is returned unrounded
    d_xy = np.empty((n, 2), dt)
    d_conic = np.empty((n, 3), dt)
    d_feat = np.empty((n, f), dt)
    d_op = np.empty((n,), dt) if op is not None else None
    args = (n, f, h, w, _p(xy), _p(conic), _p(feat), _p(op), _p(gid), _p(offs), _p(grad), _p(d_xy), _p(d_conic),
            _p(d_feat), _p(d_op), lo, hi)
    if sums == "f64":
        lib().orc_render_backward(*args)
    elif sums == "exact":
        lib().orc_render_backward_exact(*args)
    elif sums == "f64fma":
        lib().orc_render_backward_fma(*args)
    else:
        lib().orc_render_backward_f32(*args, 1 if sums == "f32r" else 0)
    return d_xy, d_conic, d_feat, d_op


def conic_to_scale_rot_grad(scale, rot, d_conic):
    scale, rot, d_conic = _f32(scale), _f32(rot), _f32(d_conic)
    n = scale.shape[0]
    d_scale = np.empty((n, 2), np.float32)
    d_rot = np.empty((n,), np.float32)
    lib().orc_conic_to_scale_rot_grad(n, _p(scale), _p(rot), _p(d_conic), _p(d_scale), _p(d_rot))
    return d_scale, d_rot


def conic_to_scale_rot_grad_f64(scale, rot, d_conic):
    """The chain rule of rasterizer_bwd.cu:128-153 evaluated in float64 (the
    truth the fp32 d_scale / d_rot are judged against)."""
    raw = np.asarray(scale, np.float64)
    th = np.asarray(rot, np.float32).astype(np.float64)
    dc = np.asarray(d_conic, np.float64)
    s = np.maximum(raw, 1e-6)
    inv2 = 1.0 / (s * s)
    diff = inv2[:, 0] - inv2[:, 1]
    c, sn = np.cos(th), np.sin(th)
    cc, ss, cs = c * c, sn * sn, c * sn
    dca, dcb, dcd = dc[:, 0], dc[:, 1], dc[:, 2]
    d_isx = cc * dca + cs * dcb + ss * dcd
    d_isy = ss * dca - cs * dcb + cc * dcd
    with np.errstate(divide="ignore", invalid="ignore"):
        d_sx = np.where(raw[:, 0] > 1e-6, d_isx * (-2.0 / raw[:, 0] ** 3), 0.0)
        d_sy = np.where(raw[:, 1] > 1e-6, d_isy * (-2.0 / raw[:, 1] ** 3), 0.0)
    d_rot = dca * (-2.0 * cs * diff) + dcb * diff * (cc - ss) + dcd * (2.0 * cs * diff)
    return np.stack([d_sx, d_sy], 1), d_rot


# the reference's fp32 evaluations the gradient bar is judged beside (render_backward sums=)
FP32_EVALUATIONS = ("f32", "f32r", "f64", "f64fma")


def grads_with_fp32_evaluation(xy, scale, rot, conic, feat, gid, offs, grad, h, w, opacity=None, tile_range=None):
    """{name: (truth, [fp32, ...])} for d_xy, d_scale, d_rot, d_feat, d_opacity
    and d_conic on the given lists: `truth` is the exact value at the fp32
    inputs (render_backward sums="exact", float64 chain rule), the parity
    target.  The list holds the reference's own fp32 arithmetic: its fp32
    per-pixel terms summed one at a time in two orders its atomics may take
    ("f32", "f32r"), summed exactly ("f64"), and with q contracted into fused
    multiply-adds as its CUDA build forms it ("f64fma"), each through the fp32
    chain rule -- the yardstick for elements whose terms cancel."""
    t = render_backward(xy, conic, feat, gid, offs, grad, h, w, opacity, tile_range, sums="exact")
    rs = [render_backward(xy, conic, feat, gid, offs, grad, h, w, opacity, tile_range, sums=k)
          for k in FP32_EVALUATIONS]
    t_scale, t_rot = conic_to_scale_rot_grad_f64(scale, rot, t[1])
    r_sr = [conic_to_scale_rot_grad(scale, rot, r[1]) for r in rs]
    out = {"d_xy": (t[0], [r[0] for r in rs]), "d_conic": (t[1], [r[1] for r in rs]),
           "d_feat": (t[2], [r[2] for r in rs]), "d_scale": (t_scale, [a for a, _ in r_sr]),
           "d_rot": (t_rot, [b for _, b in r_sr])}
    if opacity is not None:
        out["d_opacity"] = (t[3], [r[3] for r in rs])
    return out


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


# ----------------------------------------------------------------------------- feathered overlap

OVERLAP_TILE = 16


def phase_origins(overlap: int):
    """(origin_y, origin_x) of the four phase renders, oss/sr/v6/rasterizer.py:181."""
    o = int(overlap)
    return ((0, 0), (-o, 0), (0, -o), (-o, -o))


def phase_mask(h: int, w: int, origin, overlap: int) -> np.ndarray:
    """(h, w) fp32 feather weight of one phase, rasterizer.py:212-242: a cosine
    ramp over the distance of each pixel centre to the nearest tile edge of
    that phase's grid, per axis, multiplied."""
    tile = np.float32(OVERLAP_TILE)
    o = np.float32(overlap)

    def axis(n, org):
        p = np.remainder(np.arange(n, dtype=np.float32) + np.float32(0.5) - np.float32(org), tile)
        d = np.minimum(p, tile - p)
        t = np.clip(d / o, np.float32(0.0), np.float32(1.0))
        return (np.float32(0.5) - np.float32(0.5) * np.cos(t * np.float32(np.pi))).astype(np.float32)

    return (axis(h, origin[0])[:, None] * axis(w, origin[1])[None, :]).astype(np.float32)


def render_overlapped_band(xy, scale, rot, feat, opacity, h, w, overlap, rows, grad=None, mode=TIGHT):
    """The feathered 4-phase render of oss/sr/v6/rasterizer.py:159-210 over the
    output rows [rows[0], rows[1]) only: every phase renders the means
    xy - origin (fp32) on its crop rounded up to 16 with the oracle's own lists,
    the tiles covering the band are evaluated, and the crops are weighted by
    phase_mask and normalised by the weight sum (clamped at 1e-6).

    Returns {"image": (F, r1-r0, w)} and, with `grad` (F, r1-r0, w) = dL/d(band
    rows of the output, zero elsewhere), the gradients of xy, scale, rot, feat
    and opacity as {name: (truth, [fp32, ...])} pairs, as in
    grads_with_fp32_evaluation (the exact value with float64 weights, and the
    reference's fp32 arithmetic beside it)."""
    xy = _f32(xy)
    r0, r1 = int(rows[0]), int(rows[1])
    f = np.asarray(feat).shape[1]
    accum = np.zeros((f, r1 - r0, w), np.float32)
    wsum = np.zeros((r1 - r0, w), np.float32)
    phases = []
    for oy, ox in phase_origins(overlap):
        crop_h = -(-(h - min(oy, 0)) // OVERLAP_TILE) * OVERLAP_TILE
        crop_w = -(-(w - min(ox, 0)) // OVERLAP_TILE) * OVERLAP_TILE
        local = xy.copy()
        local[:, 0] = local[:, 0] - np.float32(ox)
        local[:, 1] = local[:, 1] - np.float32(oy)
        conic, _, _, gid, offs = lists(local, scale, rot, crop_h, crop_w, mode)
        ys, xs = -min(oy, 0), -min(ox, 0)
        ntx = crop_w // OVERLAP_TILE
        tr = ((r0 + ys) // OVERLAP_TILE * ntx, -(-(r1 + ys) // OVERLAP_TILE) * ntx)
        img = render_forward(local, conic, feat, gid, offs, crop_h, crop_w, opacity, tr)
        band = img[:, r0 + ys:r1 + ys, xs:xs + w]
        mask = phase_mask(h, w, (oy, ox), overlap)[r0:r1]
        accum += band * mask
        wsum += mask
        phases.append((local, conic, gid, offs, crop_h, crop_w, ys, xs, tr, mask))
    out = {"image": accum / np.maximum(wsum, np.float32(1e-6))}
    if grad is None:
        return out
    grad = np.asarray(grad, np.float32)
    wsum64 = np.zeros((r1 - r0, w), np.float64)
    for p in phases:
        wsum64 += p[-1].astype(np.float64)
    tot = {}
    for local, conic, gid, offs, crop_h, crop_w, ys, xs, tr, mask in phases:
        for kind in ("exact",) + FP32_EVALUATIONS:
            if kind in ("exact", "f64", "f64fma"):
                g_band = grad.astype(np.float64) * mask / np.maximum(wsum64, 1e-6)
            else:
                g_band = grad * (mask / np.maximum(wsum, np.float32(1e-6)))
            g_full = np.zeros((f, crop_h, crop_w), np.float32)
            g_full[:, r0 + ys:r1 + ys, xs:xs + w] = g_band.astype(np.float32)
            d = render_backward(local, conic, feat, gid, offs, g_full, crop_h, crop_w, opacity, tr, sums=kind)
            acc = tot.setdefault(kind, [np.zeros(a.shape, np.float64) if a is not None else None for a in d])
            for i, a in enumerate(d):
                if a is not None:
                    acc[i] += a
    t_xy, t_conic, t_feat, t_op = tot["exact"]
    t_scale, t_rot = conic_to_scale_rot_grad_f64(scale, rot, t_conic)
    fp32 = {"d_xy": [], "d_scale": [], "d_rot": [], "d_feat": [], "d_opacity": []}
    for kind in FP32_EVALUATIONS:
        r_xy, r_conic, r_feat, r_op = (None if a is None else a.astype(np.float32) for a in tot[kind])
        r_scale, r_rot = conic_to_scale_rot_grad(scale, rot, r_conic)
        for k, v in (("d_xy", r_xy), ("d_scale", r_scale), ("d_rot", r_rot), ("d_feat", r_feat), ("d_opacity", r_op)):
            fp32[k].append(v)
    out.update({"d_xy": (t_xy, fp32["d_xy"]), "d_scale": (t_scale, fp32["d_scale"]), "d_rot": (t_rot, fp32["d_rot"]),
                "d_feat": (t_feat, fp32["d_feat"])})
    if opacity is not None:
        out["d_opacity"] = (t_op, fp32["d_opacity"])
    return out
