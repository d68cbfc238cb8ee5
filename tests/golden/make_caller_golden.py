"""Record how the reference's own caller drives the oss_cuda op, and what it
should return.

Runs where the reference tree is importable (OSS_REFERENCE_ROOT, as
make_golden.py); writes caller_call.json and caller_cases.npz next to this
script.

    OSS_REFERENCE_ROOT=/path/to/open-supersampling python tests/golden/make_caller_golden.py

The reference's Rasterizer (oss/gaussian/renderer/rasterizer.py:142-195) is
run unchanged on fake CUDA tensors, with OSS_USE_CUDA_KERNELS set, and with a
recording module standing in for oss.cuda.oss_cuda: the record holds which
settings select the op (_custom_rasterizer_enabled, :47-52), the argument list
it passes (positional order, which GaussianBatch field each tensor is and the
operation applied to it on the way, e.g. the scale floor of :186-195) and its
return contract.  The expected images and gradients come from the same
Rasterizer with force_backend="reference" on real CPU tensors (its fp32
_render_reference, the fallback the caller would take), through autograd.
"""
from __future__ import annotations

import json
import math
import os
import sys
import types

import numpy as np
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.utils._python_dispatch import TorchDispatchMode

from make_golden import OUT, SEED, _ref_root


class _Provenance(TorchDispatchMode):
    """Remembers, for every tensor an aten op makes, the op and its inputs."""

    def __init__(self):
        super().__init__()
        self.made = {}

    def __torch_dispatch__(self, func, types_, args=(), kwargs=None):
        out = func(*args, **(kwargs or {}))
        if isinstance(out, torch.Tensor):
            self.made[id(out)] = (str(func.overloadpacket.__name__), args)
        return out


def _describe(arg, fields, prov):
    if isinstance(arg, torch.Tensor):
        for name, t in fields.items():
            if arg is t:
                return {"field": name}
        if id(arg) in prov.made:
            op, args = prov.made[id(arg)]
            return {"op": op, "args": [_describe(a, fields, prov) for a in args]}
        return {"tensor": "unknown"}
    if isinstance(arg, (bool, int, float, str)) or arg is None:
        return {"value": arg}
    return {"repr": repr(arg)}


def record_call():
    from oss.gaussian.renderer.rasterizer import GaussianBatch, Rasterizer

    calls = []
    stub = types.ModuleType("oss.cuda.oss_cuda")

    def rasterize_gaussians(*args, **kwargs):
        calls.append((args, kwargs))
        xy, feat, h, w = args[0], args[3], args[4], args[5]
        return xy.new_zeros((feat.shape[1], h, w))

    stub.rasterize_gaussians = rasterize_gaussians
    sys.modules["oss.cuda.oss_cuda"] = stub
    selects = {}
    spec = None
    for setting in ("rasterizer", "1", "true", "on", "both", "all", "rasterizer,attention", "0", "off", ""):
        os.environ["OSS_USE_CUDA_KERNELS"] = setting
        calls.clear()
        with FakeTensorMode():
            n, f, h, w = 5, 3, 40, 56
            g = GaussianBatch(xy=torch.empty(n, 2, device="cuda"), scale=torch.empty(n, 2, device="cuda"),
                              rot=torch.empty(n, device="cuda"), feat=torch.empty(n, f, device="cuda"))
            rast = Rasterizer(tile_size=16, topk_norm=True)
            backend = rast._select_backend(g)
            selects[setting] = backend == "oss_cuda"
            if backend != "oss_cuda":
                continue
            prov = _Provenance()
            with prov:
                out = rast(g, (h, w))
            args, kwargs = calls[0]
            fields = {"xy": g.xy, "scale": g.scale, "rot": g.rot, "feat": g.feat}
            this = {"args": [_describe(a, fields, prov) for a in args],
                    "kwargs": {k: _describe(v, fields, prov) for k, v in kwargs.items()},
                    "returns": [int(s) for s in out.shape], "output_hw": [h, w], "n": n, "f": f}
            assert spec is None or spec == this, "the call differs between settings"
            spec = this
    os.environ.pop("OSS_USE_CUDA_KERNELS", None)
    del sys.modules["oss.cuda.oss_cuda"]
    return {"call": spec, "selects_oss_cuda": selects,
            "source": "oss/gaussian/renderer/rasterizer.py:142-195 (Rasterizer.__call__, _select_backend, "
                      "_render_oss_cuda) run unchanged on fake CUDA tensors"}


def expected_cases():
    from oss.gaussian.renderer.rasterizer import GaussianBatch, Rasterizer

    rast = Rasterizer(tile_size=16, topk_norm=True, force_backend="reference")
    out = {}
    cases = [("a", 24, 48, 64, 3), ("b", 40, 37, 53, 5)]
    for i, (name, n, h, w, f) in enumerate(cases):
        gen = torch.Generator().manual_seed(SEED + 900 + i)
        xy = torch.rand(n, 2, generator=gen) * torch.tensor([float(w), float(h)])
        scale = torch.rand(n, 2, generator=gen) * 4.0 + 0.5
        scale[:3] = 1.0e-4  # below the caller's floor of 1e-3 (the clamp is part of the contract)
        rot = torch.rand(n, generator=gen) * math.pi
        feat = torch.randn(n, f, generator=gen)
        grad = torch.randn(f, h, w, generator=gen)
        leaves = [t.clone().requires_grad_(True) for t in (xy, scale, rot, feat)]
        img = rast(GaussianBatch(xy=leaves[0], scale=leaves[1], rot=leaves[2], feat=leaves[3]), (h, w))
        img.backward(grad)
        for k, t in zip(("xy", "scale", "rot", "feat", "grad"), (xy, scale, rot, feat, grad)):
            out[f"{name}_{k}"] = t.numpy()
        out[f"{name}_image"] = img.detach().numpy()
        for k, t in zip(("xy", "scale", "rot", "feat"), leaves):
            out[f"{name}_d_{k}"] = t.grad.numpy()
        out[f"{name}_hw"] = np.array([h, w], np.int32)
    out["names"] = np.array([c[0] for c in cases])
    return out


if __name__ == "__main__":
    sys.path.insert(0, str(_ref_root()))
    rec = record_call()
    (OUT / "caller_call.json").write_text(json.dumps(rec, indent=1) + "\n")
    np.savez_compressed(OUT / "caller_cases.npz", **expected_cases())
    print(json.dumps(rec["call"]["args"]))
    print(rec["selects_oss_cuda"])
