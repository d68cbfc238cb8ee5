"""Persistent-canvas lifecycle on the GPU (oss_b200.persistent_canvas over
csrc/canvas_life.cu) against the reference's own outputs
(tests/golden/canvas_life_cases.npz) and, at full size, against the numpy
restatement (oracle/canvas_oracle.py): index lists and slot states exactly
(modulo the reference's open order of fp32 score ties under the prune cap),
tile errors within 1e-5 abs / 1e-4 rel."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import canvas_oracle as co

pytestmark = pytest.mark.gpu

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "canvas_life_cases.npz")
KEYS = ("positions", "scales", "rotations", "colors", "age", "error", "alive")


def dev(a, dtype=None):
    t = torch.as_tensor(np.asarray(a))
    return (t.to(dtype) if dtype is not None else t).cuda().contiguous()


def host(t):
    return t.detach().cpu().numpy()


def close(got, ref, atol=1e-5, rtol=1e-4):
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=atol)


def test_tile_mse_matches_reference(cuda_device):
    from oss_b200 import per_tile_mse, per_tile_mse_lr

    for name, ts in (("mse_a", 16), ("mse_b", 8)):
        got = per_tile_mse(dev(GOLD[name + "_rendered"]), dev(GOLD[name + "_target"]), ts)
        close(host(got), GOLD[name + "_out"])
    for name in ("mse_up2", "mse_upx"):
        got = per_tile_mse_lr(dev(GOLD[name + "_rendered"]), dev(GOLD[name + "_lr"]), 16)
        close(host(got), GOLD[name + "_out"])


def test_tile_mse_full_size_against_oracle(cuda_device):
    from oss_b200 import per_tile_mse_lr

    rng = np.random.default_rng(1)
    ren = rng.random((3, 1088, 1920), dtype=np.float32)
    lr = rng.random((3, 540, 960), dtype=np.float32)
    got = host(per_tile_mse_lr(dev(ren), dev(lr), 16))
    close(got, co.per_tile_mse(ren, co.upsample_bilinear(lr, 1088, 1920), 16))


def test_tile_mse_rejects_bad_shapes(cuda_device):
    from oss_b200 import per_tile_mse

    a = torch.zeros((3, 32, 40), device="cuda")
    with pytest.raises(ValueError, match="multiples of tile_size"):
        per_tile_mse(a, a, 16)
    with pytest.raises(ValueError, match="shape mismatch"):
        per_tile_mse(torch.zeros((3, 32, 32), device="cuda"), torch.zeros((2, 32, 32), device="cuda"), 16)


def test_gaussian_error_lookup_matches_reference(cuda_device):
    from oss_b200 import gaussians_error_from_tiles

    got = gaussians_error_from_tiles(dev(GOLD["gerr_xy"]), dev(GOLD["gerr_tile"]), 16, (64, 96))
    np.testing.assert_array_equal(host(got), GOLD["gerr_out"])
    assert gaussians_error_from_tiles(torch.zeros((0, 2), device="cuda"), dev(GOLD["gerr_tile"]), 16,
                                      (64, 96)).shape == (0,)


@pytest.mark.parametrize("name", ["prune_mix", "prune_cap", "prune_pol", "prune_dead", "prune_inf"])
def test_prune_selection_matches_reference(cuda_device, name):
    from oss_b200 import PrunePolicy, select_for_pruning

    kw, okw = {}, {}
    if name + "_policy" in GOLD.files:
        p = GOLD[name + "_policy"]
        kw = dict(policy=PrunePolicy(age_max=int(p[0]), age_low_error_pct=float(p[1]), tile_error_pct=float(p[2]),
                                     min_age_before_prune=int(p[3]), max_prune_per_frame_frac=float(p[4])))
        okw = dict(age_max=int(p[0]), age_pct=float(p[1]), tile_pct=float(p[2]), min_age=int(p[3]))
    args = [GOLD[name + k] for k in ("_alive", "_in_frame", "_age", "_err")]
    got = select_for_pruning(dev(args[0]), dev(args[1]), dev(args[2]), dev(args[3]), None,
                             int(GOLD[name + "_capacity"]), **kw)
    assert got.dtype == torch.int64
    co.assert_prune_equivalent(host(got), GOLD[name + "_out"], co.prune_scores(*args, **okw))


@pytest.mark.parametrize("capacity", [10**7, 200_000, 4000])
def test_prune_selection_full_size_against_oracle(cuda_device, capacity):
    """200k slots: the quantiles, the decision tree and (for the smaller
    capacities) the cap's score order, exactly as the restatement."""
    from oss_b200 import select_for_pruning

    rng = np.random.default_rng(capacity)
    n = 200_000
    alive = rng.random(n) < 0.9
    in_frame = rng.random(n) < 0.995
    age = rng.integers(0, 100, n).astype(np.int64)
    err = rng.random(n, dtype=np.float32) * 3.0
    err[rng.random(n) < 0.01] = np.inf
    got = host(select_for_pruning(dev(alive), dev(in_frame), dev(age), dev(err), None, capacity))
    np.testing.assert_array_equal(got, co.select_for_pruning(alive, in_frame, age, err, capacity))


@pytest.mark.parametrize("k", [1, 7, 40, 200])
def test_spawn_tiles_match_reference(cuda_device, k):
    from oss_b200 import select_spawn_tiles

    st = dev(GOLD["spawn_tile"])
    np.testing.assert_array_equal(host(select_spawn_tiles(st, k)), GOLD[f"spawn_all_{k}"])
    np.testing.assert_array_equal(host(select_spawn_tiles(st, k, dev(GOLD["spawn_cls"]))), GOLD[f"spawn_cls_{k}"])


def test_spawn_tiles_full_grid_against_oracle(cuda_device):
    from oss_b200 import select_spawn_tiles

    rng = np.random.default_rng(5)
    te = rng.random((68, 120), dtype=np.float32)
    te[rng.random(te.shape) < 0.01] = np.inf
    cls = rng.random(te.shape) < 0.5
    for k in (1, 100, 5000, 10**6):
        np.testing.assert_array_equal(host(select_spawn_tiles(dev(te), k)), co.select_spawn_tiles(te, k))
        np.testing.assert_array_equal(host(select_spawn_tiles(dev(te), k, dev(cls))),
                                      co.select_spawn_tiles(te, k, cls))


def _canvas_from(prefix, capacity, feat_dim=3, hw=(32, 48), policy=None):
    from oss_b200 import PersistentCanvas

    c = PersistentCanvas(capacity=capacity, feat_dim=feat_dim, output_hw=hw, prune_policy=policy)
    c.positions = dev(GOLD[prefix + "positions"])
    c.scales = dev(GOLD[prefix + "scales"])
    c.rotations = dev(GOLD[prefix + "rotations"])
    c.colors = dev(GOLD[prefix + "colors"])
    c.age = dev(GOLD[prefix + "age"])
    c.error = dev(GOLD[prefix + "error"])
    c.alive = dev(GOLD[prefix + "alive"])
    return c


@pytest.mark.parametrize("name", ["apply_prune", "apply_more", "apply_fewer"])
def test_apply_prune_spawn_matches_reference(cuda_device, name):
    from oss_b200 import GaussianBatch, apply_prune_spawn

    c = _canvas_from(f"{name}_in_", 40)
    nb = None
    if name + "_new_xy" in GOLD.files:
        nb = GaussianBatch(*(dev(GOLD[f"{name}_new_{k}"]) for k in ("xy", "scale", "rot", "feat")))
    apply_prune_spawn(c, dev(GOLD[name + "_idx"]), nb)
    for k in KEYS:
        np.testing.assert_array_equal(host(getattr(c, k)), GOLD[f"{name}_out_{k}"], err_msg=k)


def test_apply_prune_spawn_full_size_against_oracle(cuda_device):
    from oss_b200 import GaussianBatch, PersistentCanvas, apply_prune_spawn

    rng = np.random.default_rng(8)
    n, m = 200_000, 7_000
    st = {"positions": rng.random((n, 2), dtype=np.float32), "scales": rng.random((n, 2), dtype=np.float32),
          "rotations": rng.random(n, dtype=np.float32), "colors": rng.random((n, 3), dtype=np.float32),
          "age": rng.integers(0, 50, n).astype(np.int64), "error": rng.random(n, dtype=np.float32),
          "alive": rng.random(n) < 0.97}
    idx = rng.choice(n, 9_000, replace=False).astype(np.int64)
    new = (rng.random((m, 2), dtype=np.float32), rng.random((m, 2), dtype=np.float32),
           rng.random(m, dtype=np.float32), rng.random((m, 5), dtype=np.float32))
    c = PersistentCanvas(capacity=n, feat_dim=3, output_hw=(1088, 1920))
    for k in KEYS:
        setattr(c, k, dev(st[k]))
    apply_prune_spawn(c, dev(idx), GaussianBatch(*(dev(a) for a in new)))
    ref = co.apply_prune_spawn(st, idx, new)
    for k in KEYS:
        np.testing.assert_array_equal(host(getattr(c, k)), ref[k], err_msg=k)


def test_canvas_update_frames_match_reference(cuda_device):
    """Two PersistentCanvas.update frames: warp, age, render, tile error against
    the upsampled LR frame, decision tree, spawn; slot states and statistics."""
    from oss_b200 import GaussianBatch, PrunePolicy

    c = _canvas_from("update_in_", 48, policy=PrunePolicy(age_max=2, min_age_before_prune=1,
                                                          max_prune_per_frame_frac=0.1))
    for step in range(2):
        nb = GaussianBatch(*(dev(GOLD[f"update{step}_new_{k}"]) for k in ("xy", "scale", "rot", "feat")))
        stats = c.update(dev(GOLD[f"update{step}_motion"]), dev(GOLD[f"update{step}_lr"]), new_gaussians=nb)
        ref = GOLD[f"update{step}_stats"]
        assert [stats.n_alive_before, stats.n_alive_after, stats.n_pruned, stats.n_spawned] == [int(v) for v in
                                                                                                ref[:4]]
        assert abs(stats.mean_tile_error - ref[4]) <= 1e-5 + 1e-4 * abs(ref[4])
        for k in ("scales", "rotations", "colors", "age", "alive"):
            np.testing.assert_array_equal(host(getattr(c, k)), GOLD[f"update{step}_out_{k}"], err_msg=f"{step} {k}")
        # the warped centres (grid_sample) and the tile errors to fp32 rounding
        close(host(c.positions), GOLD[f"update{step}_out_positions"])
        close(host(c.error), GOLD[f"update{step}_out_error"])


def test_canvas_rejects_cpu_and_bad_arguments():
    from oss_b200 import PersistentCanvas

    with pytest.raises(ValueError, match="capacity must be positive"):
        PersistentCanvas(capacity=0)
    with pytest.raises(ValueError, match="multiples of tile_size"):
        PersistentCanvas(capacity=4, output_hw=(30, 32), device="cuda")
    with pytest.raises(RuntimeError, match="CUDA"):
        PersistentCanvas(capacity=4, output_hw=(32, 32), device="cpu")
