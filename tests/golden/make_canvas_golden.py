"""Golden vectors of the persistent canvas's lifecycle from the reference's own
PyTorch code (oss/gaussian/canvas/{error_detection,prune_spawn,canvas,warp}.py).

Runs only where the reference tree is importable (OSS_REFERENCE_ROOT, as for
make_golden.py); the output is the committed fixture canvas_life_cases.npz,
which the tests read instead of the reference.

    OSS_REFERENCE_ROOT=/path/to/open-supersampling python tests/golden/make_canvas_golden.py

Cases
  mse_*      per_tile_mse on (F, H, W) pairs, and on a render against an LR frame
             bilinearly upsampled by F.interpolate (integer and non-integer ratios).
  gerr_*     gaussians_error_from_tiles with centres on tile edges, on the frame
             border and outside it.
  prune_*    select_for_pruning: a mixed scene under the default policy, the
             per-frame cap (out-of-frame ties and priority order), a custom policy,
             an all-dead canvas and alive +inf errors.
  spawn_*    select_spawn_tiles with and without a classifier mask and +inf tiles.
  apply_*    apply_prune_spawn on a small canvas (prune only, prune + spawn with
             more and with fewer replacements than free slots).
  update_*   two PersistentCanvas.update frames on a 48-slot canvas (render by the
             reference rasterizer), every state array and statistic after each.
Inputs avoid exact ties where the reference leaves an order open (topk and the
cap's argsort), except the out-of-frame ties, which its stable sort fixes.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "canvas_life_cases.npz"


def main() -> None:
    root = os.environ.get("OSS_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set OSS_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, str(Path(root)))
    import torch.nn.functional as F
    from oss.gaussian.canvas.canvas import PersistentCanvas
    from oss.gaussian.canvas.error_detection import gaussians_error_from_tiles, per_tile_mse
    from oss.gaussian.canvas.prune_spawn import (PrunePolicy, apply_prune_spawn, select_for_pruning,
                                                 select_spawn_tiles)
    from oss.gaussian.renderer import GaussianBatch

    torch.manual_seed(0)
    g = torch.Generator().manual_seed(0x5EED)
    out = {}

    # ---- per-tile MSE
    r = torch.rand(3, 64, 96, generator=g)
    t = torch.rand(3, 64, 96, generator=g)
    out["mse_a_rendered"], out["mse_a_target"] = r.numpy(), t.numpy()
    out["mse_a_out"] = per_tile_mse(r, t, 16).numpy()
    r1 = torch.rand(1, 32, 32, generator=g) * 4.0
    t1 = torch.rand(1, 32, 32, generator=g)
    out["mse_b_rendered"], out["mse_b_target"] = r1.numpy(), t1.numpy()
    out["mse_b_out"] = per_tile_mse(r1, t1, 8).numpy()
    for name, (h, w) in (("mse_up2", (32, 48)), ("mse_upx", (23, 37))):
        lr = torch.rand(3, h, w, generator=g)
        ren = torch.rand(3, 64, 96, generator=g)
        up = F.interpolate(lr.unsqueeze(0), size=(64, 96), mode="bilinear", align_corners=False).squeeze(0)
        out[name + "_lr"], out[name + "_rendered"] = lr.numpy(), ren.numpy()
        out[name + "_out"] = per_tile_mse(ren, up, 16).numpy()

    # ---- per-Gaussian error lookup
    te = torch.rand(4, 6, generator=g)
    xy = torch.rand(200, 2, generator=g) * torch.tensor([110.0, 76.0]) - torch.tensor([7.0, 6.0])
    xy[:8] = torch.tensor([[0.0, 0.0], [95.9999, 63.9999], [96.0, 10.0], [10.0, 64.0], [-1e-6, 5.0],
                           [16.0, 16.0], [15.99999, 31.99999], [47.5, 0.0]])
    out["gerr_tile"], out["gerr_xy"] = te.numpy(), xy.numpy()
    out["gerr_out"] = gaussians_error_from_tiles(xy, te, 16, (64, 96)).numpy()

    # ---- prune selection
    def prune_case(name, n, alive_p, frame_p, err, age_hi, capacity, policy=None):
        alive = torch.rand(n, generator=g) < alive_p
        in_frame = torch.rand(n, generator=g) < frame_p
        age = torch.randint(0, age_hi, (n,), generator=g)
        idx = select_for_pruning(alive, in_frame, age, err, None, capacity, policy)
        out[name + "_alive"], out[name + "_in_frame"] = alive.numpy(), in_frame.numpy()
        out[name + "_age"], out[name + "_err"] = age.numpy(), err.numpy()
        out[name + "_capacity"] = np.array(capacity)
        out[name + "_out"] = idx.numpy()
        if policy is not None:
            out[name + "_policy"] = np.array([policy.age_max, policy.age_low_error_pct, policy.tile_error_pct,
                                              policy.min_age_before_prune, policy.max_prune_per_frame_frac])

    prune_case("prune_mix", 500, 0.9, 0.97, torch.rand(500, generator=g), 120, 20000)
    prune_case("prune_cap", 400, 0.95, 0.8, torch.rand(400, generator=g), 120, 400)
    prune_case("prune_pol", 300, 0.8, 0.95, torch.rand(300, generator=g) * 10.0, 40, 3000,
               PrunePolicy(age_max=10, age_low_error_pct=0.5, tile_error_pct=0.8, min_age_before_prune=1,
                           max_prune_per_frame_frac=0.1))
    prune_case("prune_dead", 64, 0.0, 0.5, torch.rand(64, generator=g), 120, 64)
    e = torch.rand(256, generator=g)
    e[::9] = float("inf")
    prune_case("prune_inf", 256, 0.9, 1.0, e, 120, 4000)

    # ---- spawn tiles
    st = torch.rand(8, 12, generator=g)
    st[2, 3] = float("inf")
    cls = torch.rand(8, 12, generator=g) < 0.6
    out["spawn_tile"], out["spawn_cls"] = st.numpy(), cls.numpy()
    for k in (1, 7, 40, 200):
        out[f"spawn_all_{k}"] = select_spawn_tiles(st, k).numpy()
        out[f"spawn_cls_{k}"] = select_spawn_tiles(st, k, cls).numpy()

    # ---- apply prune / spawn
    def small_canvas(cap):
        c = PersistentCanvas(capacity=cap, feat_dim=3, output_hw=(32, 48))
        c.positions = torch.rand(cap, 2, generator=g) * 40.0
        c.scales = torch.rand(cap, 2, generator=g) + 0.5
        c.rotations = torch.rand(cap, generator=g) * 3.0
        c.colors = torch.rand(cap, 3, generator=g)
        c.age = torch.randint(0, 50, (cap,), generator=g)
        c.error = torch.rand(cap, generator=g)
        c.alive = torch.rand(cap, generator=g) < 0.8
        return c

    def batch(m, f):
        return GaussianBatch(xy=torch.rand(m, 2, generator=g) * 40.0, scale=torch.rand(m, 2, generator=g) + 0.5,
                             rot=torch.rand(m, generator=g) * 3.0, feat=torch.rand(m, f, generator=g))

    for name, m, f in (("apply_prune", None, 0), ("apply_more", 30, 3), ("apply_fewer", 2, 5)):
        c = small_canvas(40)
        for key in ("positions", "scales", "rotations", "colors", "age", "error", "alive"):
            out[f"{name}_in_{key}"] = getattr(c, key).numpy().copy()
        idx = torch.tensor([3, 0, 17, 39, 22])
        nb = batch(m, f) if m is not None else None
        if nb is not None:
            out[f"{name}_new_xy"], out[f"{name}_new_scale"] = nb.xy.numpy(), nb.scale.numpy()
            out[f"{name}_new_rot"], out[f"{name}_new_feat"] = nb.rot.numpy(), nb.feat.numpy()
        out[f"{name}_idx"] = idx.numpy()
        apply_prune_spawn(c, idx, nb)
        for key in ("positions", "scales", "rotations", "colors", "age", "error", "alive"):
            out[f"{name}_out_{key}"] = getattr(c, key).numpy().copy()

    # ---- two update frames
    c = PersistentCanvas(capacity=48, feat_dim=3, output_hw=(32, 48),
                         prune_policy=PrunePolicy(age_max=2, min_age_before_prune=1, max_prune_per_frame_frac=0.1))
    c.initialize_random(seed=11)
    c.scales = torch.rand(48, 2, generator=g) * 3.0 + 1.0
    c.rotations = torch.rand(48, generator=g) * 3.0
    c.colors = torch.rand(48, 3, generator=g)
    c.alive[::7] = False
    for key in ("positions", "scales", "rotations", "colors", "age", "error", "alive"):
        out[f"update_in_{key}"] = getattr(c, key).numpy().copy()
    yy, xx = torch.meshgrid(torch.arange(32.0), torch.arange(48.0), indexing="ij")
    for step in range(2):
        motion = torch.stack([3.0 * torch.sin(yy / 9.0 + step), 2.0 * torch.cos(xx / 13.0 - step)]) * (1 + step)
        lr = torch.rand(3, 16, 24, generator=g)
        nb = batch(6, 3)
        out[f"update{step}_motion"], out[f"update{step}_lr"] = motion.numpy(), lr.numpy()
        out[f"update{step}_new_xy"], out[f"update{step}_new_scale"] = nb.xy.numpy(), nb.scale.numpy()
        out[f"update{step}_new_rot"], out[f"update{step}_new_feat"] = nb.rot.numpy(), nb.feat.numpy()
        stats = c.update(motion, lr, new_gaussians=nb)
        out[f"update{step}_stats"] = np.array([stats.n_alive_before, stats.n_alive_after, stats.n_pruned,
                                               stats.n_spawned, stats.mean_tile_error])
        for key in ("positions", "scales", "rotations", "colors", "age", "error", "alive"):
            out[f"update{step}_out_{key}"] = getattr(c, key).numpy().copy()

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({len(out)} arrays)")


if __name__ == "__main__":
    main()
