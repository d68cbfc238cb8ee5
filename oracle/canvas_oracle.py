"""CPU restatement (numpy) of the persistent canvas's lifecycle steps -- TEST
INFRASTRUCTURE ONLY: the checker of liboss_b200.so's canvas kernels, imported by
tests/ and never by the product path.

Pinned against tests/golden/canvas_life_cases.npz (outputs of the reference's
own code, made by tests/golden/make_canvas_golden.py) in
tests/test_oracle_canvas.py.  Each function cites the reference lines it follows.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def upsample_bilinear(lr: np.ndarray, h: int, w: int) -> np.ndarray:
    """F.interpolate(bilinear, align_corners=False) of (F, hl, wl) to (F, h, w)
    (the LR frame of oss/gaussian/canvas/canvas.py:256-263): source coordinate
    (dst + 0.5) * in / out - 0.5 clamped at 0, neighbours clamped at the edge."""
    f, hl, wl = lr.shape
    if (hl, wl) == (h, w):
        return lr.astype(F32)

    def axis(n_out, n_in):
        s = F32(F32(n_in) / F32(n_out))
        src = (np.arange(n_out, dtype=F32) + F32(0.5)) * s - F32(0.5)
        src = np.maximum(src, F32(0.0)).astype(F32)
        i0 = src.astype(np.int64)
        i1 = np.where(i0 < n_in - 1, i0 + 1, i0)
        l1 = (src - i0.astype(F32)).astype(F32)
        return i0, i1, l1, (F32(1.0) - l1).astype(F32)

    y0, y1, ly1, ly0 = axis(h, hl)
    x0, x1, lx1, lx0 = axis(w, wl)
    a = lr.astype(F32)
    top = lx0[None, None, :] * a[:, y0][:, :, x0] + lx1[None, None, :] * a[:, y0][:, :, x1]
    bot = lx0[None, None, :] * a[:, y1][:, :, x0] + lx1[None, None, :] * a[:, y1][:, :, x1]
    return (ly0[None, :, None] * top + ly1[None, :, None] * bot).astype(F32)


def per_tile_mse(rendered: np.ndarray, target: np.ndarray, ts: int) -> np.ndarray:
    """error_detection.py:26-63: channel mean of the squared difference, then
    the mean over each ts x ts tile (float64 sums)."""
    f, h, w = rendered.shape
    sq = ((rendered.astype(np.float64) - target.astype(np.float64)) ** 2).mean(axis=0)
    return sq.reshape(h // ts, ts, w // ts, ts).mean(axis=(1, 3)).astype(F32)


def gaussians_error_from_tiles(xy: np.ndarray, tile_err: np.ndarray, ts: int, hw) -> np.ndarray:
    """error_detection.py:66-113: the error of the tile holding the centre,
    +inf outside [0, W) x [0, H)."""
    H, W = hw
    h, w = tile_err.shape
    x, y = xy[:, 0].astype(F32), xy[:, 1].astype(F32)
    with np.errstate(invalid="ignore"):
        inside = (x >= 0) & (x < F32(W)) & (y >= 0) & (y < F32(H))
        tx = np.clip(np.trunc(np.where(inside, x, 0) / F32(ts)).astype(np.int64), 0, w - 1)
        ty = np.clip(np.trunc(np.where(inside, y, 0) / F32(ts)).astype(np.int64), 0, h - 1)
    return np.where(inside, tile_err[ty, tx], F32(np.inf)).astype(F32)


def _fma32(a, b, c):
    return F32(np.float64(a) * np.float64(b) + np.float64(c))


def quantile(x: np.ndarray, q: float) -> np.float32:
    """torch.quantile (linear) as the reference calls it (prune_spawn.py:111-125):
    fp32 rank q * (m - 1), neighbours of the ascending sort (NaN last) and
    torch's lerp, whose two fused multiply-adds start from the nearer end; NaN
    if any value is NaN."""
    v = np.sort(x.astype(F32))
    m = v.size
    if np.isnan(v[-1]):
        return F32(np.nan)
    r = F32(F32(q) * F32(m - 1))
    lo, hi = int(r), int(np.ceil(r))
    wgt = F32(r - F32(lo))
    a, b = v[lo], v[hi]
    with np.errstate(invalid="ignore", over="ignore"):
        d = F32(b - a)
        if wgt < 0.5:
            return _fma32(wgt, d, a)
        return _fma32(-d, F32(1.0) - wgt, b)


def select_for_pruning(alive, in_frame, age, err, capacity, age_max=60, age_pct=0.75, tile_pct=0.95, min_age=3,
                       frac=0.05) -> np.ndarray:
    """prune_spawn.py:72-157: R1 | R2 | R3 in slot order; above the cap
    max(1, int(frac * capacity)) the cap's worth by priority * 1e6 + error
    (non-finite as 1e30) descending, ties in slot order."""
    alive = alive.astype(bool)
    in_frame = in_frame.astype(bool)
    err = err.astype(F32)
    n = alive.size
    if n == 0:
        return np.zeros((0,), np.int64)
    live = err[alive]
    age_q = quantile(live, age_pct) if live.size else F32(0.0)
    tile_q = quantile(live, tile_pct) if live.size else F32(np.inf)
    with np.errstate(invalid="ignore"):
        r1 = alive & ~in_frame
        r2 = alive & (age > age_max) & (err <= age_q)
        r3 = alive & (age >= min_age) & (err >= tile_q)
    sel = np.flatnonzero(r1 | r2 | r3)
    cap = max(1, int(frac * capacity))
    if sel.size <= cap:
        return sel.astype(np.int64)
    prio = np.where(r1, F32(3), np.where(r2, F32(2), np.where(r3, F32(1), F32(0)))).astype(F32)[sel]
    e = err[sel]
    clipped = np.where(np.isfinite(e), e, F32(1e30)).astype(F32)
    score = (prio * F32(1e6)).astype(F32) + clipped
    order = np.argsort(-score.astype(np.float64), kind="stable")
    return sel[order[:cap]].astype(np.int64)


def prune_scores(alive, in_frame, age, err, age_max=60, age_pct=0.75, tile_pct=0.95, min_age=3) -> np.ndarray:
    """The cap's sort key per slot (priority * 1e6 + clipped error, fp32), as
    select_for_pruning computes it (prune_spawn.py:139-152)."""
    alive = alive.astype(bool)
    in_frame = in_frame.astype(bool)
    err = err.astype(F32)
    live = err[alive]
    age_q = quantile(live, age_pct) if live.size else F32(0.0)
    tile_q = quantile(live, tile_pct) if live.size else F32(np.inf)
    with np.errstate(invalid="ignore"):
        r1 = alive & ~in_frame
        r2 = alive & (age > age_max) & (err <= age_q)
        r3 = alive & (age >= min_age) & (err >= tile_q)
    prio = np.where(r1, F32(3), np.where(r2, F32(2), np.where(r3, F32(1), F32(0)))).astype(F32)
    clipped = np.where(np.isfinite(err), err, F32(1e30)).astype(F32)
    return ((prio * F32(1e6)).astype(F32) + clipped).astype(F32)


def select_spawn_tiles(tile_err: np.ndarray, n_tiles: int, cls=None) -> np.ndarray:
    """prune_spawn.py:165-208: (ty, tx) of the largest errors (classifier-masked
    tiles at -inf, NaN largest, ties in tile order), min(n_tiles, finite
    eligible) of them."""
    h, w = tile_err.shape
    v = tile_err.astype(F32) if cls is None else np.where(cls, tile_err, F32(-np.inf)).astype(F32)
    flat = v.ravel()
    take = min(int(n_tiles), int(np.isfinite(flat).sum()))
    if take <= 0:
        return np.zeros((0, 2), np.int64)
    key = np.where(np.isnan(flat), np.inf, flat.astype(np.float64))
    order = np.argsort(-key, kind="stable")[:take]
    return np.stack([order // w, order % w], axis=-1).astype(np.int64)


def apply_prune_spawn(state: dict, prune_idx: np.ndarray, new=None) -> dict:
    """prune_spawn.py:216-255 on a dict of canvas arrays (positions, scales,
    rotations, colors, age, error, alive); new = (xy, scale, rot, feat) or None."""
    s = {k: v.copy() for k, v in state.items()}
    if prune_idx.size:
        s["alive"][prune_idx] = False
        s["age"][prune_idx] = 0
        s["error"][prune_idx] = 0.0
    if new is None:
        return s
    xy, scale, rot, feat = new
    free = np.flatnonzero(~s["alive"])
    m = min(free.size, xy.shape[0])
    wr = free[:m]
    s["positions"][wr] = xy[:m]
    s["scales"][wr] = scale[:m]
    s["rotations"][wr] = rot[:m]
    f = min(s["colors"].shape[1], feat.shape[1])
    s["colors"][wr, :f] = feat[:m, :f]
    s["alive"][wr] = True
    s["age"][wr] = 0
    s["error"][wr] = 0.0
    return s


def assert_prune_equivalent(got, ref, score):
    """Equal lists, except where the reference's cap cut an fp32 score tie: its
    argsort leaves the order of equal keys open (and priority * 1e6 + error
    rounds errors to multiples of 0.25), where these keep slot order.  Then the
    same length, descending scores, the same multiset of scores and every slot
    scored above the last one kept."""
    got, ref = np.asarray(got), np.asarray(ref)
    if np.array_equal(got, ref):
        return
    assert got.size == ref.size
    sg, sr = score[got], score[ref]
    assert np.all(np.diff(sg.astype(np.float64)) <= 0) and np.all(np.diff(sr.astype(np.float64)) <= 0)
    np.testing.assert_array_equal(np.sort(sg), np.sort(sr))
    cut = sr[-1]
    assert set(np.flatnonzero(score > cut)) <= set(got.tolist()) & set(ref.tolist())
