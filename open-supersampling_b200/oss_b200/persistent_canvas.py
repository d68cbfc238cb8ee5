"""The persistent canvas's per-frame lifecycle on the B200 kernels.

Drop-in for oss/gaussian/canvas/canvas.py (``PersistentCanvas``, ``CanvasStats``),
oss/gaussian/canvas/error_detection.py (``per_tile_mse``,
``gaussians_error_from_tiles``) and oss/gaussian/canvas/prune_spawn.py
(``PrunePolicy``, ``select_for_pruning``, ``select_spawn_tiles``,
``apply_prune_spawn``): the same signatures, shapes, dtypes and error
messages.  Each step is a call into liboss_b200.so (csrc/canvas_life.cu): the
tile error (with the LR frame's bilinear upsample fused in), the per-slot
error and age, the decision tree's quantiles and its per-frame cap, the
spawn-tile ranking and the slot update all run on the device; a function
that returns a variable-length tensor reads its length once, as nonzero()
does in the reference.

Where the reference leaves an order open (ties in the cap's argsort and in
topk) these functions keep slot / tile order.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch

from oss_cuda import _lib
from oss_cuda._raster import stream_of

from .v6 import render as _render
from .warp import warp_positions

__all__ = ["CanvasStats", "GaussianBatch", "PersistentCanvas", "PrunePolicy", "apply_prune_spawn",
           "gaussians_error_from_tiles", "per_tile_mse", "per_tile_mse_lr", "select_for_pruning",
           "select_spawn_tiles"]


@dataclass
class GaussianBatch:
    """SoA batch of 2D Gaussians (oss/gaussian/renderer/rasterizer.py:56-99)."""

    xy: torch.Tensor
    scale: torch.Tensor
    rot: torch.Tensor
    feat: torch.Tensor

    def __post_init__(self) -> None:
        n = self.xy.shape[0]
        if self.xy.shape != (n, 2):
            raise ValueError(f"xy must be (N, 2), got {tuple(self.xy.shape)}")
        if self.scale.shape != (n, 2):
            raise ValueError(f"scale must be (N, 2), got {tuple(self.scale.shape)}")
        if self.rot.shape != (n,):
            raise ValueError(f"rot must be (N,), got {tuple(self.rot.shape)}")
        if self.feat.ndim != 2 or self.feat.shape[0] != n:
            raise ValueError(f"feat must be (N, F), got {tuple(self.feat.shape)}")
        for name, t in (("xy", self.xy), ("scale", self.scale), ("rot", self.rot), ("feat", self.feat)):
            if t.device != self.xy.device:
                raise ValueError(f"all tensors must share a device; {name} on {t.device}, xy on {self.xy.device}")

    @property
    def num_gaussians(self) -> int:
        return self.xy.shape[0]

    @property
    def feat_dim(self) -> int:
        return self.feat.shape[1]

    @property
    def device(self) -> torch.device:
        return self.xy.device


def _cuda(t: torch.Tensor, name: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor (the canvas lifecycle runs on liboss_b200.so)")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.float32).contiguous()


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.uint8).contiguous()


def _scratch(nbytes: int, device) -> torch.Tensor:
    return torch.empty((max(1, int(nbytes)),), device=device, dtype=torch.uint8)


# ---------------------------------------------------------------------------
# Error detection (error_detection.py)
# ---------------------------------------------------------------------------


def _tile_mse(rendered: torch.Tensor, target: torch.Tensor, tile_size: int) -> torch.Tensor:
    f, H, W = rendered.shape
    lib = _lib.lib()
    r, t = _f32(rendered), _f32(target)
    with torch.cuda.device(rendered.device):
        out = torch.empty((H // tile_size, W // tile_size), device=rendered.device, dtype=torch.float32)
        _lib.check(lib.oss_tile_mse(f, H, W, tile_size, r.data_ptr(), t.shape[1], t.shape[2], t.data_ptr(),
                                    out.data_ptr(), stream_of(r)), "oss_tile_mse")
    return out.to(rendered.dtype)


def per_tile_mse(rendered: torch.Tensor, lr_upsampled: torch.Tensor, tile_size: int = 16) -> torch.Tensor:
    """Mean squared error per ``tile_size x tile_size`` tile, averaged over
    channels (error_detection.py:26-63): (F, H, W) x 2 -> (H/ts, W/ts)."""
    if rendered.shape != lr_upsampled.shape:
        raise ValueError(f"rendered {tuple(rendered.shape)} vs lr_upsampled {tuple(lr_upsampled.shape)} shape mismatch")
    if rendered.ndim != 3:
        raise ValueError(f"rendered must be (F, H, W); got {tuple(rendered.shape)}")
    _, H, W = rendered.shape
    if H % tile_size or W % tile_size:
        raise ValueError(f"H={H} W={W} must both be multiples of tile_size={tile_size}")
    _cuda(rendered, "rendered")
    return _tile_mse(rendered, lr_upsampled, tile_size)


def per_tile_mse_lr(rendered: torch.Tensor, lr_frame: torch.Tensor, tile_size: int = 16) -> torch.Tensor:
    """per_tile_mse against ``lr_frame`` (F, h, w) bilinearly upsampled to the
    render's size (F.interpolate, align_corners=False; canvas.py:256-263), with
    the upsample done inside the tile kernel."""
    if rendered.ndim != 3 or lr_frame.ndim != 3 or lr_frame.shape[0] != rendered.shape[0]:
        raise ValueError(f"rendered {tuple(rendered.shape)} and lr_frame {tuple(lr_frame.shape)} must be (F, H, W)"
                         " with the same F")
    _, H, W = rendered.shape
    if H % tile_size or W % tile_size:
        raise ValueError(f"H={H} W={W} must both be multiples of tile_size={tile_size}")
    _cuda(rendered, "rendered")
    return _tile_mse(rendered, lr_frame, tile_size)


def gaussians_error_from_tiles(xy: torch.Tensor, tile_err: torch.Tensor, tile_size: int,
                               hw: Tuple[int, int]) -> torch.Tensor:
    """Per-Gaussian error = that of the tile holding its centre; +inf outside
    the frame (error_detection.py:66-113)."""
    if xy.ndim != 2 or xy.shape[1] != 2:
        raise ValueError(f"xy must be (N, 2); got {tuple(xy.shape)}")
    if tile_err.ndim != 2:
        raise ValueError(f"tile_err must be (h, w); got {tuple(tile_err.shape)}")
    H, W = hw
    h, w = tile_err.shape
    if h * tile_size != H or w * tile_size != W:
        raise ValueError(f"tile_err {tile_err.shape} * tile_size={tile_size} != hw={hw}")
    n = xy.shape[0]
    if n == 0:
        return torch.zeros((0,), dtype=tile_err.dtype, device=tile_err.device)
    _cuda(xy, "xy")
    p, te = _f32(xy), _f32(tile_err)
    with torch.cuda.device(xy.device):
        out = torch.empty((n,), device=xy.device, dtype=torch.float32)
        _lib.check(_lib.lib().oss_canvas_error(n, H, W, tile_size, p.data_ptr(), None, te.data_ptr(), None, None,
                                               out.data_ptr(), None, stream_of(p)), "oss_canvas_error")
    return out.to(tile_err.dtype)


# ---------------------------------------------------------------------------
# Prune / spawn (prune_spawn.py)
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class PrunePolicy:
    """Thresholds of the prune decision tree (prune_spawn.py:36-62)."""

    age_max: int = 60
    age_low_error_pct: float = 0.75
    tile_error_pct: float = 0.95
    min_age_before_prune: int = 3
    max_prune_per_frame_frac: float = 0.05


def _prune_device(alive, in_frame, age, g_error, capacity, p):
    """Device-side decision tree: (prune_idx[n] int64, count int64[1], quantiles[2])."""
    n = alive.shape[0]
    dev = alive.device
    lib = _lib.lib()
    idx = torch.empty((max(1, n),), device=dev, dtype=torch.int64)
    cnt = torch.empty((1,), device=dev, dtype=torch.int64)
    quant = torch.empty((2,), device=dev, dtype=torch.float32)
    scratch = _scratch(lib.oss_prune_scratch_bytes(n), dev)
    with torch.cuda.device(dev):
        _lib.check(lib.oss_select_for_pruning(n, _lib.ptr(alive), _lib.ptr(in_frame), _lib.ptr(age),
                                               _lib.ptr(g_error), int(capacity), int(p.age_max),
                                               float(p.age_low_error_pct), float(p.tile_error_pct),
                                               int(p.min_age_before_prune), float(p.max_prune_per_frame_frac),
                                               idx.data_ptr(), cnt.data_ptr(), quant.data_ptr(), scratch.data_ptr(),
                                               scratch.numel(), stream_of(alive)), "oss_select_for_pruning")
    return idx, cnt, quant


def select_for_pruning(alive_mask: torch.Tensor, in_frame: torch.Tensor, age: torch.Tensor, g_error: torch.Tensor,
                       tile_error: torch.Tensor, capacity: int, policy: Optional[PrunePolicy] = None) -> torch.Tensor:
    """Long indices of the slots to retire this frame (prune_spawn.py:72-157):
    R1 alive and out of frame; R2 older than age_max with error at or below the
    age quantile of the alive errors; R3 at least min_age_before_prune old with
    error at or above the tile quantile; at most max(1, floor(frac * capacity)),
    then by priority (R1 > R2 > R3) and error."""
    p = policy if policy is not None else PrunePolicy()
    n = alive_mask.shape[0]
    if n == 0:
        return torch.zeros((0,), dtype=torch.long, device=alive_mask.device)
    _cuda(alive_mask, "alive_mask")
    idx, cnt, _ = _prune_device(_u8(alive_mask), _u8(in_frame), age.detach().to(torch.int64).contiguous(),
                                _f32(g_error), capacity, p)
    return idx[: int(cnt.item())].clone()


def select_spawn_tiles(tile_error: torch.Tensor, n_tiles: int,
                       classifier_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(M, 2) long (y, x) of the top-error tiles, restricted to classifier_mask
    (prune_spawn.py:165-208)."""
    if tile_error.ndim != 2:
        raise ValueError(f"tile_error must be (h, w); got {tuple(tile_error.shape)}")
    h, w = tile_error.shape
    if classifier_mask is not None and classifier_mask.shape != tile_error.shape:
        raise ValueError(f"classifier_mask {classifier_mask.shape} != tile_error {tile_error.shape}")
    dev = tile_error.device
    if h * w == 0:
        return torch.zeros((0, 2), dtype=torch.long, device=dev)
    _cuda(tile_error, "tile_error")
    lib = _lib.lib()
    te = _f32(tile_error)
    cls = _u8(classifier_mask) if classifier_mask is not None else None
    out = torch.empty((h * w, 2), device=dev, dtype=torch.int64)
    take = torch.empty((1,), device=dev, dtype=torch.int64)
    scratch = _scratch(lib.oss_spawn_tiles_scratch_bytes(h * w), dev)
    with torch.cuda.device(dev):
        _lib.check(lib.oss_select_spawn_tiles(h, w, te.data_ptr(), _lib.ptr(cls), int(n_tiles), out.data_ptr(),
                                              take.data_ptr(), scratch.data_ptr(), scratch.numel(), stream_of(te)),
                   "oss_select_spawn_tiles")
    return out[: int(take.item())].clone()


def _apply_device(canvas, idx, cnt, max_prune, new_gaussians):
    """Device-side slot update; returns the spawned count as a device int64[1]."""
    lib = _lib.lib()
    n = canvas.capacity
    dev = canvas.device
    spawned = torch.empty((1,), device=dev, dtype=torch.int64)
    scratch = _scratch(lib.oss_prune_spawn_scratch_bytes(n), dev)
    if new_gaussians is not None and new_gaussians.num_gaussians > 0:
        gb = new_gaussians
        nxy, nsc, nrot, nfeat = _f32(gb.xy), _f32(gb.scale), _f32(gb.rot), _f32(gb.feat)
        m, f_new = gb.num_gaussians, gb.feat_dim
    else:
        nxy = nsc = nrot = nfeat = None
        m, f_new = 0, 0
    with torch.cuda.device(dev):
        _lib.check(lib.oss_apply_prune_spawn(n, canvas.feat_dim, _lib.ptr(idx), _lib.ptr(cnt), int(max_prune), m,
                                             f_new, _lib.ptr(nxy), _lib.ptr(nsc), _lib.ptr(nrot), _lib.ptr(nfeat),
                                             canvas.positions.data_ptr(), canvas.scales.data_ptr(),
                                             canvas.rotations.data_ptr(), canvas.colors.data_ptr(),
                                             canvas.alive.data_ptr(), canvas.age.data_ptr(), canvas.error.data_ptr(),
                                             spawned.data_ptr(), scratch.data_ptr(), scratch.numel(),
                                             stream_of(canvas.positions)), "oss_apply_prune_spawn")
    return spawned


def apply_prune_spawn(canvas: "PersistentCanvas", prune_idx: torch.Tensor,
                      new_gaussians: Optional[GaussianBatch] = None) -> None:
    """Mark ``prune_idx`` dead (age and error reset), then write ``new_gaussians``
    into the dead slots in slot order, as many as fit (prune_spawn.py:216-255)."""
    k = int(prune_idx.numel())
    idx = cnt = None
    if k > 0:
        lo, hi = int(prune_idx.min()), int(prune_idx.max())
        if lo < -canvas.capacity or hi >= canvas.capacity:
            raise IndexError(f"index out of range for a canvas of capacity {canvas.capacity}")
        idx = torch.remainder(prune_idx.detach().to(device=canvas.device, dtype=torch.int64), canvas.capacity)
        cnt = torch.tensor([k], device=canvas.device, dtype=torch.int64)
    if k == 0 and new_gaussians is None:
        return
    _apply_device(canvas, idx, cnt, k, new_gaussians)


# ---------------------------------------------------------------------------
# The canvas (canvas.py)
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class CanvasStats:
    """One update's diagnostics (canvas.py:43-51)."""

    n_alive_before: int
    n_alive_after: int
    n_pruned: int
    n_spawned: int
    mean_tile_error: float


class PersistentCanvas:
    """Persistent SoA canvas warped by motion each frame, with per-tile error
    driving prune and spawn (canvas.py:54-298).  CUDA only: its storage lives
    on the device and every step of ``update`` runs in liboss_b200.so."""

    def __init__(self, capacity: int = 8000, feat_dim: int = 3, output_hw: Tuple[int, int] = (720, 1280),
                 tile_size: int = 16, device: torch.device | str = "cuda", dtype: torch.dtype = torch.float32,
                 prune_policy: Optional[PrunePolicy] = None) -> None:
        if capacity <= 0:
            raise ValueError(f"capacity must be positive; got {capacity}")
        if feat_dim <= 0:
            raise ValueError(f"feat_dim must be positive; got {feat_dim}")
        h, w = output_hw
        if h <= 0 or w <= 0:
            raise ValueError(f"output_hw must be positive; got {output_hw}")
        if h % tile_size or w % tile_size:
            raise ValueError(f"output_hw {output_hw} must be multiples of tile_size={tile_size}")
        if dtype != torch.float32:
            raise ValueError("the device canvas stores float32")
        self.capacity = int(capacity)
        self.feat_dim = int(feat_dim)
        self.output_hw = (int(h), int(w))
        self.tile_size = int(tile_size)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("PersistentCanvas runs on liboss_b200.so and needs a CUDA device")
        self.dtype = dtype
        self.policy = prune_policy if prune_policy is not None else PrunePolicy()
        self.positions = torch.zeros((capacity, 2), dtype=dtype, device=self.device)
        self.scales = torch.ones((capacity, 2), dtype=dtype, device=self.device)
        self.rotations = torch.zeros((capacity,), dtype=dtype, device=self.device)
        self.colors = torch.zeros((capacity, feat_dim), dtype=dtype, device=self.device)
        self.age = torch.zeros((capacity,), dtype=torch.long, device=self.device)
        self.error = torch.zeros((capacity,), dtype=dtype, device=self.device)
        self.alive = torch.zeros((capacity,), dtype=torch.bool, device=self.device)

    def initialize_random(self, seed: Optional[int] = None) -> None:
        """Random Gaussians over the frame, half-tile scale, colour 0.5 (canvas.py:122-142)."""
        gen = torch.Generator(device="cpu")
        if seed is not None:
            gen.manual_seed(int(seed))
        h, w = self.output_hw
        xs = torch.rand((self.capacity,), generator=gen) * w
        ys = torch.rand((self.capacity,), generator=gen) * h
        self.positions[:, 0] = xs.to(self.dtype).to(self.device)
        self.positions[:, 1] = ys.to(self.dtype).to(self.device)
        self.scales[:, :] = float(self.tile_size) * 0.5
        self.rotations[:] = 0.0
        self.colors[:] = 0.5
        self.age[:] = 0
        self.error[:] = 0.0
        self.alive[:] = True

    def initialize_from_batch(self, batch: GaussianBatch) -> None:
        """Seed from a batch; extra slots stay dead (canvas.py:144-158)."""
        n = min(batch.num_gaussians, self.capacity)
        self.alive[:] = False
        self.age[:] = 0
        self.error[:] = 0.0
        self.positions[:n] = batch.xy[:n].to(self.positions.dtype).to(self.device)
        self.scales[:n] = batch.scale[:n].to(self.scales.dtype).to(self.device)
        self.rotations[:n] = batch.rot[:n].to(self.rotations.dtype).to(self.device)
        f = min(self.feat_dim, batch.feat_dim)
        self.colors[:n, :f] = batch.feat[:n, :f].to(self.colors.dtype).to(self.device)
        self.alive[:n] = True

    @property
    def n_alive(self) -> int:
        return int(self.alive.sum().item())

    def snapshot(self) -> GaussianBatch:
        """The alive subset as a renderer-ready batch (canvas.py:166-175)."""
        idx = self.alive.nonzero(as_tuple=False).flatten()
        return GaussianBatch(xy=self.positions[idx], scale=self.scales[idx], rot=self.rotations[idx],
                             feat=self.colors[idx])

    def render(self) -> torch.Tensor:
        """(F, H, W) render of the alive Gaussians (canvas.py:177-189)."""
        gb = self.snapshot()
        if gb.num_gaussians == 0:
            return torch.zeros((self.feat_dim, *self.output_hw), dtype=self.dtype, device=self.device)
        h, w = self.output_hw
        return _render(gb.xy.contiguous(), gb.scale.contiguous(), gb.rot.contiguous(), gb.feat.contiguous(), h, w)

    def update(self, motion: torch.Tensor, lr_frame: torch.Tensor, new_gaussians: Optional[GaussianBatch] = None,
               classifier_mask: Optional[torch.Tensor] = None) -> CanvasStats:
        """One frame (canvas.py:191-295): warp the positions, bump the ages,
        render, score the tiles against the upsampled LR frame, give every slot
        its tile's error, prune and write the replacements.  The host waits
        three times: for the alive list and the pair total of the render, and for
        the statistics at the end.  The reference also ranks spawn tiles here and
        discards the ranking (canvas.py:281-289); ``classifier_mask`` only feeds
        that ranking, so it is accepted and unused (``select_spawn_tiles`` gives
        the ranking to callers that want it)."""
        H, W = self.output_hw
        T = self.tile_size
        new_xy, in_frame = warp_positions(self.positions, motion, self.output_hw)
        self.positions = new_xy.contiguous()
        n_before = torch.count_nonzero(self.alive)
        rendered = self.render()
        if lr_frame.ndim != 3 or lr_frame.shape[0] != rendered.shape[0]:
            raise ValueError(f"lr_frame must be (F, h, w) with F={rendered.shape[0]}; got {tuple(lr_frame.shape)}")
        tile_err = per_tile_mse_lr(rendered, lr_frame, T)
        alive_u8 = self.alive.view(torch.uint8)
        frame_u8 = _u8(in_frame)
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            _lib.check(lib.oss_canvas_error(self.capacity, H, W, T, self.positions.data_ptr(), frame_u8.data_ptr(),
                                            tile_err.data_ptr(), alive_u8.data_ptr(), self.age.data_ptr(), None,
                                            self.error.data_ptr(), stream_of(self.positions)), "oss_canvas_error")
        idx, cnt, _ = _prune_device(alive_u8, frame_u8, self.age, self.error, self.capacity, self.policy)
        _apply_device(self, idx, cnt, self.capacity, new_gaussians)
        stats = torch.stack([n_before.to(torch.float64), torch.count_nonzero(self.alive).to(torch.float64),
                             cnt[0].to(torch.float64), tile_err.to(torch.float64).mean()]).tolist()
        n_pruned = int(stats[2])
        return CanvasStats(n_alive_before=int(stats[0]), n_alive_after=int(stats[1]), n_pruned=n_pruned,
                           n_spawned=min(new_gaussians.num_gaussians, n_pruned) if new_gaussians is not None else 0,
                           mean_tile_error=float(np.float32(stats[3])))
