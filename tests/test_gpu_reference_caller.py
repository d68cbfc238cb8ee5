"""The reference's caller, replayed against this package.

tests/golden/make_caller_golden.py ran the reference's Rasterizer
(oss/gaussian/renderer/rasterizer.py:142-195) unchanged with
OSS_USE_CUDA_KERNELS set and recorded the call it makes into oss_cuda
(caller_call.json): which settings select the op, the positional argument
list (which GaussianBatch field each tensor is, and the scale floor applied on
the way) and the returned shape.  Here that exact call goes to this package's
oss_cuda.rasterize_gaussians, and its image and gradients are held to the
parity bar against what the same Rasterizer returns with its reference backend
(caller_cases.npz, from the reference's autograd).
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import oracle as orc
from conftest import GOLDEN, assert_close, assert_close_grad, golden_case, load_golden

CALL = json.loads((GOLDEN / "caller_call.json").read_text())


def _replay(arg, fields, h, w, index, spec):
    if "field" in arg:
        return fields[arg["field"]]
    if "op" in arg:
        inputs = [_replay(a, fields, h, w, -1, spec) for a in arg["args"]]
        return getattr(torch, arg["op"])(*inputs)
    if "value" in arg:
        # the recorded output size stands for this case's (h, w)
        if index in (4, 5) and arg["value"] == spec["output_hw"][index - 4]:
            return (h, w)[index - 4]
        return arg["value"]
    raise AssertionError(f"unreplayable argument {arg}")


def test_recorded_call_is_the_drop_in_contract():
    spec = CALL["call"]
    assert [a.get("field") for a in spec["args"][:4]] == ["xy", None, "rot", "feat"]
    assert spec["args"][1] == {"op": "clamp_min", "args": [{"field": "scale"}, {"value": 0.001}]}
    assert spec["args"][6:] == [{"value": 16}, {"value": True}] and spec["kwargs"] == {}
    assert spec["returns"] == [spec["f"], *spec["output_hw"]]
    assert all(CALL["selects_oss_cuda"][k] for k in ("rasterizer", "1", "true", "on", "both", "all"))
    assert not any(CALL["selects_oss_cuda"][k] for k in ("0", "off", ""))


@pytest.mark.gpu
def test_reference_caller_call_matches_reference_backend(cuda_device):
    import oss_cuda
    from oss_cuda import rasterizer

    assert rasterizer._COMPILED
    spec = CALL["call"]
    data = load_golden("caller_cases.npz")
    for name in data["names"]:
        c = golden_case(data, str(name))
        h, w = (int(v) for v in c["hw"])
        leaves = {k: torch.from_numpy(c[k]).to(cuda_device).requires_grad_(True) for k in ("xy", "scale", "rot", "feat")}
        args = [_replay(a, leaves, h, w, i, spec) for i, a in enumerate(spec["args"])]
        out = oss_cuda.rasterize_gaussians(*args)
        assert tuple(out.shape) == (c["feat"].shape[1], h, w)
        assert_close(out.detach().cpu().numpy(), c["image"], what=f"{name} image")
        out.backward(torch.from_numpy(c["grad"]).to(cuda_device))
        # the exact gradients of the same render (oracle, scale floored as the caller does), with
        # the reference backend's fp32 autograd values among the fp32 evaluations
        floored = np.maximum(c["scale"], np.float32(1e-3))
        conic, _, _, gid, offs = orc.lists(c["xy"], floored, c["rot"], h, w, orc.EXACT)
        ref = orc.grads_with_fp32_evaluation(c["xy"], floored, c["rot"], conic, c["feat"], gid, offs, c["grad"],
                                             h, w)
        ref["d_scale"] = tuple(np.where(c["scale"] >= 1e-3, v, 0.0) if i == 0 else
                               [np.where(c["scale"] >= 1e-3, r, 0.0) for r in v] for i, v in enumerate(ref["d_scale"]))
        for k, t in leaves.items():
            truth, fp32 = ref[f"d_{k}" if k != "feat" else "d_feat"]
            assert_close_grad(t.grad.cpu().numpy(), truth, what=f"{name} d_{k}", ref32=fp32 + [c[f"d_{k}"]])
            assert_close_grad(c[f"d_{k}"], truth, what=f"{name} reference backend d_{k}", ref32=fp32 + [c[f"d_{k}"]])
        # the floor: Gaussians below it get no scale gradient, as under the reference's clamp
        assert np.all(leaves["scale"].grad.cpu().numpy()[:3] == 0.0)
