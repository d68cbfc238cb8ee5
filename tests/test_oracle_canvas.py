"""The numpy restatement of the canvas lifecycle (oracle/canvas_oracle.py)
against the reference's own outputs (tests/golden/canvas_life_cases.npz, made
by tests/golden/make_canvas_golden.py): tile errors to fp32 rounding, every
index list and state array exactly."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import canvas_oracle as co

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "canvas_life_cases.npz")


def test_per_tile_mse_matches_reference():
    for name, ts in (("mse_a", 16), ("mse_b", 8)):
        got = co.per_tile_mse(GOLD[name + "_rendered"], GOLD[name + "_target"], ts)
        np.testing.assert_allclose(got, GOLD[name + "_out"], rtol=2e-6, atol=0)


@pytest.mark.parametrize("name", ["mse_up2", "mse_upx"])
def test_upsampled_tile_mse_matches_reference(name):
    ren = GOLD[name + "_rendered"]
    up = co.upsample_bilinear(GOLD[name + "_lr"], ren.shape[1], ren.shape[2])
    np.testing.assert_allclose(co.per_tile_mse(ren, up, 16), GOLD[name + "_out"], rtol=2e-6, atol=0)


def test_gaussian_error_lookup_matches_reference():
    got = co.gaussians_error_from_tiles(GOLD["gerr_xy"], GOLD["gerr_tile"], 16, (64, 96))
    np.testing.assert_array_equal(got, GOLD["gerr_out"])


@pytest.mark.parametrize("name", ["prune_mix", "prune_cap", "prune_pol", "prune_dead", "prune_inf"])
def test_prune_selection_matches_reference(name):
    kw = {}
    if name + "_policy" in GOLD.files:
        p = GOLD[name + "_policy"]
        kw = dict(age_max=int(p[0]), age_pct=float(p[1]), tile_pct=float(p[2]), min_age=int(p[3]), frac=float(p[4]))
    args = (GOLD[name + "_alive"], GOLD[name + "_in_frame"], GOLD[name + "_age"], GOLD[name + "_err"])
    got = co.select_for_pruning(*args, int(GOLD[name + "_capacity"]), **kw)
    co.assert_prune_equivalent(got, GOLD[name + "_out"], co.prune_scores(*args, **{k: v for k, v in kw.items()
                                                                             if k != "frac"}))


@pytest.mark.parametrize("k", [1, 7, 40, 200])
def test_spawn_tiles_match_reference(k):
    np.testing.assert_array_equal(co.select_spawn_tiles(GOLD["spawn_tile"], k), GOLD[f"spawn_all_{k}"])
    np.testing.assert_array_equal(co.select_spawn_tiles(GOLD["spawn_tile"], k, GOLD["spawn_cls"]),
                                  GOLD[f"spawn_cls_{k}"])


@pytest.mark.parametrize("name", ["apply_prune", "apply_more", "apply_fewer"])
def test_apply_prune_spawn_matches_reference(name):
    keys = ("positions", "scales", "rotations", "colors", "age", "error", "alive")
    state = {k: GOLD[f"{name}_in_{k}"] for k in keys}
    new = None
    if name + "_new_xy" in GOLD.files:
        new = tuple(GOLD[f"{name}_new_{k}"] for k in ("xy", "scale", "rot", "feat"))
    got = co.apply_prune_spawn(state, GOLD[name + "_idx"], new)
    for k in keys:
        np.testing.assert_array_equal(got[k], GOLD[f"{name}_out_{k}"], err_msg=k)


def test_quantile_restatement_edge_cases():
    """Single value, exact ranks, +inf neighbours (NaN from the lerp, as torch
    gives) and NaN inputs."""
    assert co.quantile(np.array([2.5], np.float32), 0.95) == np.float32(2.5)
    assert co.quantile(np.array([0, 1, 2, 3, 4], np.float32), 0.75) == np.float32(3.0)
    assert co.quantile(np.array([0, 1, np.inf], np.float32), 0.5) == np.float32(1.0)
    # an infinite upper neighbour: weight >= 1/2 gives fma(-inf, 1 - w, inf) = NaN, below it inf
    assert np.isnan(co.quantile(np.array([0, 1, np.inf], np.float32), 0.75))
    assert co.quantile(np.array([0, 1, np.inf], np.float32), 0.6) == np.float32(np.inf)
    assert co.quantile(np.array([0, 1, np.inf], np.float32), 0.4) == np.float32(0.8)
    assert np.isnan(co.quantile(np.array([0, np.nan, 1], np.float32), 0.1))
