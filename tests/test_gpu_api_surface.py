"""The build-added surface of the drop-in package: rasterize_gaussians'
overlap / phase_offset keywords, rasterize_gaussians_batched and
warp_canvas_cuda, each checked bit for bit against the composition it stands
for (whose parity the other GPU tests pin against the oracle)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _gaussians(n, h, w, f, seed):
    rng = np.random.default_rng(seed)
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    scale = np.exp(rng.standard_normal((n, 2)) * 0.3 + math.log(2.0)).astype(np.float32)
    rot = (rng.random(n) * math.pi).astype(np.float32)
    feat = rng.random((n, f)).astype(np.float32)
    opacity = (1.0 / (1.0 + np.exp(-rng.standard_normal(n)))).astype(np.float32)
    return [torch.from_numpy(a).cuda() for a in (xy, scale, rot, feat, opacity)]


def _leaves(ts):
    return [t.detach().clone().requires_grad_(True) for t in ts]


@pytest.mark.parametrize("binning,h,w,f,capacity", [
    ("tight3sigma", 80, 112, 3, None),
    ("exact", 80, 112, 3, None),
    ("exact56", 83, 97, 3, None),  # ragged last tile row and column of every frame
    ("tight3sigma", 83, 97, 5, None),
    ("tight3sigma", 80, 112, 3, 20_000),  # sync-free: the device checks the capacity
])
def test_batched_equals_per_frame_calls(cuda_device, binning, h, w, f, capacity):
    """One launch chain over the frames (stacked tile grid) against one call per
    frame: images and gradients bit for bit."""
    from oss_cuda import pair_capacity_overflowed, rasterize_gaussians, rasterize_gaussians_batched

    sizes = [300, 0, 517, 64]
    offs = [0]
    for s in sizes:
        offs.append(offs[-1] + s)
    xy, scale, rot, feat, op = _gaussians(offs[-1], h, w, f, 3)
    grad = torch.randn((len(sizes), f, h, w), device="cuda")
    a = _leaves((xy, scale, rot, feat, op))
    pair_capacity_overflowed()
    img = rasterize_gaussians_batched(a[0], a[1], a[2], a[3], offs, h, w, binning=binning, opacity=a[4],
                                      pair_capacity=capacity)
    assert not pair_capacity_overflowed()
    assert img.shape == (len(sizes), f, h, w)
    img.backward(grad)
    b = _leaves((xy, scale, rot, feat, op))
    for i, (lo, hi) in enumerate(zip(offs, offs[1:])):
        one = rasterize_gaussians(b[0][lo:hi], b[1][lo:hi], b[2][lo:hi], b[3][lo:hi], h, w, binning=binning,
                                  opacity=b[4][lo:hi])
        assert torch.equal(one.detach(), img[i].detach())
        one.backward(grad[i])
    for x, y in zip(a, b):
        assert torch.equal(x.grad, y.grad)


@pytest.mark.parametrize("sizes", [[700], [0, 0, 400], [250, 0], [37] * 12])
def test_batched_edge_frames(cuda_device, sizes):
    """One frame, leading and trailing empty frames, a frame whose Gaussians all
    lie outside it, many small frames: the one-chain batch equals the per-frame
    calls bit for bit."""
    from oss_cuda import rasterize_gaussians, rasterize_gaussians_batched

    h, w = 48, 80
    offs = [0]
    for s_ in sizes:
        offs.append(offs[-1] + s_)
    xy, scale, rot, feat, op = _gaussians(offs[-1], h, w, 3, 17)
    if len(sizes) > 1 and sizes[0] > 0:
        xy[: sizes[0]] += torch.tensor([3.0 * w, 0.0], device="cuda")  # the first frame's Gaussians off screen
    grad = torch.randn((len(sizes), 3, h, w), device="cuda")
    a = _leaves((xy, scale, rot, feat, op))
    img = rasterize_gaussians_batched(a[0], a[1], a[2], a[3], offs, h, w, binning="tight3sigma", opacity=a[4])
    img.backward(grad)
    b = _leaves((xy, scale, rot, feat, op))
    for i, (lo, hi) in enumerate(zip(offs, offs[1:])):
        one = rasterize_gaussians(b[0][lo:hi], b[1][lo:hi], b[2][lo:hi], b[3][lo:hi], h, w, binning="tight3sigma",
                                  opacity=b[4][lo:hi])
        assert torch.equal(one.detach(), img[i].detach())
        one.backward(grad[i])
    for x, y in zip(a, b):
        assert torch.equal(x.grad, y.grad)


def test_batched_many_frames(cuda_device):
    """40 frames of 270x480 (20,400 tiles in the stacked grid: the tile-offset scan
    takes its per-block sums first) against per-frame calls, images and gradients
    bit for bit."""
    from oss_cuda import rasterize_gaussians, rasterize_gaussians_batched

    h, w, frames, per = 270, 480, 40, 500
    offs = [f * per for f in range(frames + 1)]
    xy, scale, rot, feat, op = _gaussians(offs[-1], h, w, 3, 23)
    grad = torch.randn((frames, 3, h, w), device="cuda")
    a = _leaves((xy, scale, rot, feat, op))
    img = rasterize_gaussians_batched(a[0], a[1], a[2], a[3], offs, h, w, binning="exact56", opacity=a[4])
    img.backward(grad)
    b = _leaves((xy, scale, rot, feat, op))
    for i, (lo, hi) in enumerate(zip(offs, offs[1:])):
        one = rasterize_gaussians(b[0][lo:hi], b[1][lo:hi], b[2][lo:hi], b[3][lo:hi], h, w, binning="exact56",
                                  opacity=b[4][lo:hi])
        assert torch.equal(one.detach(), img[i].detach())
        one.backward(grad[i])
    for x, y in zip(a, b):
        assert torch.equal(x.grad, y.grad)


def test_batched_capacity_overflow_zeroes_and_flags(cuda_device):
    from oss_cuda import pair_capacity_overflowed, rasterize_gaussians_batched

    h, w = 64, 96
    xy, scale, rot, feat, op = _gaussians(900, h, w, 3, 19)
    pair_capacity_overflowed()
    img = rasterize_gaussians_batched(xy, scale, rot, feat, [0, 450, 900], h, w, binning="tight3sigma",
                                      opacity=op, pair_capacity=10)
    assert pair_capacity_overflowed()
    assert not img.any()


def test_batched_graph_outlives_offset_cache_eviction(cuda_device):
    """A graph captured with one frame split still renders it after 70 other
    splits have passed through the offsets cache: the captured split's device
    tensor is kept, the uncaptured ones are dropped beyond 64."""
    from oss_cuda import _batched, rasterize_gaussians_batched

    h, w, n = 48, 64, 600
    xy, scale, rot, feat, op = _gaussians(n, h, w, 3, 29)
    offs = [0, 250, n]
    kw = dict(binning="tight3sigma", opacity=op, pair_capacity=20_000)
    want = rasterize_gaussians_batched(xy, scale, rot, feat, offs, h, w, **kw)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        rasterize_gaussians_batched(xy, scale, rot, feat, offs, h, w, **kw)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        got = rasterize_gaussians_batched(xy, scale, rot, feat, offs, h, w, **kw)
    for k in range(70):
        rasterize_gaussians_batched(xy, scale, rot, feat, [0, 100 + k, n], h, w, **kw)
    key = (torch.cuda.current_device(), tuple(offs))
    assert key in _batched._FRAME_OFFSETS
    assert sum(k not in _batched._CAPTURED for k in _batched._FRAME_OFFSETS) <= _batched._MAX_UNCAPTURED
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    del graph


def test_batched_rejects_bad_offsets(cuda_device):
    from oss_cuda import rasterize_gaussians_batched

    xy, scale, rot, feat, _ = _gaussians(10, 32, 32, 3, 1)
    for offs in ([0, 5], [1, 10], [0, 6, 4, 10]):
        with pytest.raises(ValueError):
            rasterize_gaussians_batched(xy, scale, rot, feat, offs, 32, 32)


def test_phase_offset_is_a_shift_of_the_means(cuda_device):
    from oss_cuda import rasterize_gaussians

    h, w = 64, 96
    xy, scale, rot, feat, op = _gaussians(700, h, w, 3, 5)
    a = _leaves((xy, scale, rot, feat))
    img = rasterize_gaussians(*a, h, w, binning="tight3sigma", phase_offset=(5, -3))
    img.sum().backward()
    b = _leaves((xy, scale, rot, feat))
    ref = rasterize_gaussians(b[0] + torch.tensor([5.0, -3.0], device="cuda"), b[1], b[2], b[3], h, w,
                              binning="tight3sigma")
    ref.sum().backward()
    assert torch.equal(img.detach(), ref.detach())
    for x, y in zip(a, b):
        assert torch.equal(x.grad, y.grad)


def test_overlap_keyword_is_the_feathered_render(cuda_device):
    from oss_b200 import render_overlapped
    from oss_cuda import rasterize_gaussians

    h, w = 70, 90
    xy, scale, rot, feat, op = _gaussians(600, h, w, 4, 7)
    a = _leaves((xy, scale, rot, feat))
    img = rasterize_gaussians(*a, h, w, binning="tight3sigma", overlap=4)
    img.sum().backward()
    b = _leaves((xy, scale, rot, feat))
    ref = render_overlapped(*b, h, w, 4, "tight3sigma")  # scales are far above its 1e-3 floor
    ref.sum().backward()
    assert torch.equal(img.detach(), ref.detach())
    for x, y in zip(a, b):
        assert torch.equal(x.grad, y.grad)
    with pytest.raises(ValueError):
        rasterize_gaussians(*a, h, w, overlap=-1)
    with pytest.raises(ValueError):
        rasterize_gaussians(*a, h, w, overlap=4, blend="alpha", opacity=op)


def test_warp_canvas_cuda_is_the_canvas_warp(cuda_device):
    from oss_b200 import CanvasState, warp_canvas
    from oss_cuda import warp_canvas_cuda

    n, h, w = 500, 96, 128
    g = torch.Generator(device="cuda").manual_seed(9)
    canvas = CanvasState(torch.rand((n, 2), device="cuda", generator=g) * torch.tensor([w, h], device="cuda"),
                         torch.rand((n, 2), device="cuda", generator=g) + 0.5,
                         torch.rand((n,), device="cuda", generator=g) * 3.0,
                         torch.rand((n,), device="cuda", generator=g),
                         torch.rand((n, 3), device="cuda", generator=g), count=n)
    motion = (torch.rand((1, 2, h // 2, w // 2), device="cuda", generator=g) - 0.5) * 8.0
    a = warp_canvas_cuda(canvas, motion, (h, w), sigma_recon=0.5, alpha=0.5)
    b = warp_canvas(canvas, motion, (h, w), sigma_recon=0.5, alpha=0.5)
    assert a.count == b.count
    for x, y in zip((a.positions, a.scales, a.rotations, a.opacities, a.colors),
                    (b.positions, b.scales, b.rotations, b.opacities, b.colors)):
        assert torch.equal(x, y)


def test_render_canvas_at_lr_is_the_scaled_weight_sum_render(cuda_device):
    """The LR render for ConcatFusion (oss/sr/v6/model.py:628-678): the canvas
    divided by the upscale factor through V6Rasterizer with the weight-sum
    channel, expanded over the batch; zeros without a canvas."""
    from oss_b200 import CanvasState, V6Rasterizer, render_canvas_at_lr

    n, h_lr, w_lr, s = 800, 48, 80, 2.0
    g = torch.Generator(device="cuda").manual_seed(4)
    canvas = CanvasState(torch.rand((n, 2), device="cuda", generator=g) * torch.tensor([w_lr * s, h_lr * s],
                                                                                       device="cuda"),
                         torch.rand((n, 2), device="cuda", generator=g) * 3.0 + 1.0,
                         torch.rand((n,), device="cuda", generator=g) * 3.0,
                         torch.rand((n,), device="cuda", generator=g),
                         torch.rand((n, 8), device="cuda", generator=g), count=n)
    ras = V6Rasterizer(token_dim=32, latent_rank=8)
    mask = torch.rand((n,), device="cuda", generator=g) > 0.3
    G, m = render_canvas_at_lr(ras, canvas, mask, 2, h_lr, w_lr, s, torch.device("cuda"), torch.float32)
    assert G.shape == (2, 8, h_lr, w_lr) and m.shape == (2, 1, h_lr, w_lr)
    scaled = CanvasState(canvas.positions / s, canvas.scales / s, canvas.rotations, canvas.opacities,
                         canvas.colors, count=n)
    G2, m2 = ras(scaled, mask.unsqueeze(0).expand(2, -1), output_hw=(h_lr, w_lr), return_weight_sum=True)
    assert torch.equal(G, G2) and torch.equal(m, m2)
    assert float(m.max()) > 0.0
    Gz, mz = render_canvas_at_lr(ras, None, None, 3, h_lr, w_lr, s, torch.device("cuda"), torch.float32)
    assert Gz.shape == (3, 8, h_lr, w_lr) and not Gz.any() and not mz.any()


def test_rasterize_gaussians_compiles_fullgraph(cuda_device):
    """torch.compile(fullgraph=True) traces a loss through rasterize_gaussians
    (the render is one dispatcher-visible operator, oss_cuda.ops) and gives
    the eager loss and gradients."""
    from conftest import assert_close
    from oss_cuda import rasterize_gaussians

    rng = np.random.default_rng(17)
    n, h, w = 2000, 96, 160
    xy = torch.from_numpy((rng.random((n, 2)) * np.array([w, h])).astype(np.float32)).to(cuda_device)
    scale = torch.from_numpy(np.exp(rng.standard_normal((n, 2)) * 0.3 + 0.7).astype(np.float32)).to(cuda_device)
    rot = torch.from_numpy((rng.random(n) * 3.1).astype(np.float32)).to(cuda_device)
    rgb = torch.from_numpy(rng.random((n, 3)).astype(np.float32)).to(cuda_device)
    op = torch.from_numpy(rng.random(n).astype(np.float32)).to(cuda_device)
    target = torch.from_numpy(rng.random((3, h, w)).astype(np.float32)).to(cuda_device)

    def loss_fn(xy, scale, rot, rgb, op):
        img = rasterize_gaussians(xy, scale, rot, rgb, h, w, binning="tight3sigma", opacity=op)
        return ((img - target) ** 2).mean()

    def run(fn):
        leaves = [t.clone().requires_grad_(True) for t in (xy, scale, rot, rgb, op)]
        loss = fn(*leaves)
        loss.backward()
        return loss.detach(), [t.grad for t in leaves]

    torch._dynamo.reset()
    compiled = torch.compile(loss_fn, fullgraph=True)
    l_c, g_c = run(compiled)
    l_e, g_e = run(loss_fn)
    assert torch.allclose(l_c, l_e, rtol=1e-6, atol=1e-7)
    for a, b in zip(g_c, g_e):
        assert_close(a.cpu().numpy(), b.cpu().numpy(), what="compiled gradient")
