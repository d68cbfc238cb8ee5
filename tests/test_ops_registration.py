"""The dispatcher-visible operators (oss_cuda.ops): registered under
torch.ops.oss_b200, with fake kernels that give torch.compile the output
shapes without a device, and an autograd formula.  CPU-only checks; the
compiled-versus-eager comparison runs on the GPU (test_gpu_api_surface)."""
from __future__ import annotations

import torch
from torch._subclasses.fake_tensor import FakeTensorMode


def test_ops_are_registered():
    import oss_cuda  # noqa: F401  (registers the operators)

    assert hasattr(torch.ops.oss_b200, "rasterize_sum")
    assert hasattr(torch.ops.oss_b200, "rasterize_sum_backward")


def test_fake_kernels_give_the_shapes():
    import oss_cuda  # noqa: F401

    n, f, h, w = 7, 3, 20, 36
    with FakeTensorMode():
        xy, scale, rot = torch.empty(n, 2), torch.empty(n, 2), torch.empty(n)
        feat, op, grad = torch.empty(n, f), torch.empty(n), torch.empty(f, h, w)
        img = torch.ops.oss_b200.rasterize_sum(xy, scale, rot, feat, op, h, w, 0, -1)
        assert tuple(img.shape) == (f, h, w)
        d = torch.ops.oss_b200.rasterize_sum_backward(xy, scale, rot, feat, op, grad, h, w, 0, -1)
        assert [tuple(t.shape) for t in d] == [(n, 2), (n, 2), (n,), (n, f), (n,)]
        d = torch.ops.oss_b200.rasterize_sum_backward(xy, scale, rot, feat, None, grad, h, w, 0, -1)
        assert tuple(d[4].shape) == (0,)
