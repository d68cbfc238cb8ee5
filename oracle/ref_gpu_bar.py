"""Time the reference's own CUDA op (oracle/_ref/_C.so, built for sm_100a by
build_ref.py) beside the product on the same B200 and the same seeded inputs.

TEST INFRASTRUCTURE: a kernel-level speed bar, not the product.  Prints one
JSON line per measurement.  Inputs stay resident on the device; every timed
iteration starts after a 256 MB L2 flush and is bracketed by CUDA events on
the current stream.

What the reference's public op does (oss/cuda/oss_cuda/rasterizer.py:28-70):
``_C.rasterize_forward`` builds full-frame tile lists (every Gaussian in every
tile, rasterizer_fwd.cu:547-564) and sums them with a bf16-split wmma kernel;
the backward runs over those same lists with per-pixel float atomics
(rasterizer_bwd.cu:32-113).  That is timed as ``ref_live``.  Its 3-sigma list
builder ``_C.pair_construction_only`` (torch sort of 64-bit keys) feeding its
backward kernel is timed as ``ref_tight`` (the forward kernel is not callable
on custom lists through the reference's API).

    python oracle/ref_gpu_bar.py [--configs 1,2] [--iters 3]
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent / "open-supersampling_b200"))

CONFIGS = {
    # BASELINE configs 1 and 2: (h, w, n, log-scale mean)
    1: (540, 960, 16384, math.log(1.5)),
    2: (1080, 1920, 200000, math.log(2.0)),
}


def make_inputs(cfg, dev, seed=0):
    h, w, n, mu = CONFIGS[cfg]
    rng = np.random.default_rng(seed)
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    scale = np.exp(rng.standard_normal((n, 2)) * 0.3 + mu).astype(np.float32)
    rot = (rng.random(n) * math.pi).astype(np.float32)
    opacity = (1.0 / (1.0 + np.exp(-rng.standard_normal(n)))).astype(np.float32)
    rgb = rng.random((n, 3)).astype(np.float32)
    feat = rgb * opacity[:, None]  # opacity folded into the summed features, as the reference's callers do
    grad = rng.standard_normal((3, h, w)).astype(np.float32)
    t = [torch.from_numpy(a).to(dev).contiguous() for a in (xy, scale, rot, feat, grad)]
    return h, w, n, t


def timed(fn, iters, flush):
    fn()  # warm-up
    torch.cuda.synchronize()
    ms = []
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    return float(np.median(ms)), ms


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--configs", default="1,2")
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()

    import build_ref
    from oss_cuda import _C as ours
    from oss_cuda import rasterize_gaussians

    ref = build_ref.load_built()
    dev = torch.device("cuda:0")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def emit(**kv):
        print(json.dumps(kv), flush=True)

    for cfg in [int(c) for c in args.configs.split(",")]:
        h, w, n, (xy, scale, rot, feat, grad) = make_inputs(cfg, dev)
        px = h * w

        def line(what, impl, ms, samples, extra=None):
            emit(config=cfg, what=what, impl=impl, ms=round(ms, 4), mpix_per_s=round(px / (ms * 1e3), 2),
                 samples_ms=[round(s, 4) for s in samples], **(extra or {}))

        # --- forward, the public op -------------------------------------------------------
        ms, s = timed(lambda: ref.rasterize_forward(xy, scale, rot, feat, h, w, 16, True), args.iters, flush)
        line("fwd", "ref_live (full-frame lists, bf16-split wmma)", ms, s)
        for binning in ("exact", "tight3sigma"):
            ms, s = timed(lambda: ours.rasterize_forward(xy, scale, rot, feat, h, w, 16, True, binning=binning),
                          args.iters, flush)
            line("fwd", f"b200 ({binning} lists)", ms, s)

        # --- image agreement on this input --------------------------------------------------
        out_r = ref.rasterize_forward(xy, scale, rot, feat, h, w, 16, True)[0]
        out_k = ours.rasterize_forward(xy, scale, rot, feat, h, w, 16, True, binning="exact")[0]
        err = (out_k - out_r).abs()
        emit(config=cfg, what="image max|b200 exact - ref_live|", value=float(err.max()),
             ref_max=float(out_r.abs().max()))
        del out_r, out_k

        # --- fwd + bwd --------------------------------------------------------------------------
        def ref_live_step():
            out, g, off, conic = ref.rasterize_forward(xy, scale, rot, feat, h, w, 16, True)
            d_xy, d_conic, d_feat = ref.rasterize_backward(xy, scale, rot, feat, conic, g, off, grad, h, w, 16)
            ref.conic_to_scale_rot_grad(scale, rot, d_conic)

        if cfg == 1:  # O(N x tiles x 256) float atomics: config 1 only
            ms, s = timed(ref_live_step, args.iters, flush)
            line("fwd+bwd", "ref_live (full-frame lists, per-pixel atomics)", ms, s)

        g_t, off_t, conic_t, tot_t = ref.pair_construction_only(xy, scale, rot, h, w, 16)
        ms, s = timed(lambda: ref.pair_construction_only(xy, scale, rot, h, w, 16), args.iters, flush)
        line("binning", "ref pair_construction_only (3-sigma, torch sort)", ms, s, {"pairs": int(tot_t)})
        ms, s = timed(lambda: ref.rasterize_backward(xy, scale, rot, feat, conic_t, g_t, off_t, grad, h, w, 16),
                      args.iters, flush)
        line("bwd", "ref_tight (3-sigma lists, per-pixel atomics)", ms, s, {"pairs": int(tot_t)})
        ms, s = timed(lambda: ours.rasterize_backward(xy, scale, rot, feat, conic_t, g_t, off_t, grad, h, w, 16),
                      args.iters, flush)
        line("bwd", "b200 rasterize_backward (same 3-sigma lists)", ms, s, {"pairs": int(tot_t)})

        for binning in ("exact", "tight3sigma"):
            leaves = [t.detach().clone().requires_grad_(True) for t in (xy, scale, rot, feat)]

            def step():
                for t in leaves:
                    t.grad = None
                out = rasterize_gaussians(*leaves, h, w, binning=binning)
                out.backward(grad)

            ms, s = timed(step, args.iters, flush)
            line("fwd+bwd", f"b200 rasterize_gaussians autograd ({binning} lists)", ms, s)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
