"""Parity against the reference's own CUDA extension on the same B200.

oracle/build_ref.py compiles the reference's four op sources
(oss/cuda/src/{bindings.cpp,rasterizer_fwd.cu,rasterizer_bwd.cu,
tile_bin_counting_sort.cu}) for sm_100a into oracle/_ref/_C.so.  Every test
here calls the six entry points of that module and of the product's
``oss_cuda._C`` with the same tensors and compares the results with the bars
the reference's own GPU tests use (tests/cuda/test_preprocess_kernel.py:43-45,
test_pair_construction_kernel.py:59-62, test_rasterizer_equivalence.py:53,
test_rasterizer_backward_equivalence.py:71-95):

* conic 1e-6, AABBs, pair counts and tile lists bit-exact;
* forward images 5e-3: the reference's forward feeds weights and features to
  bf16 tensor-core MMAs as hi/lo pairs, so it is itself only 5e-3-close to its
  fp32 definition (the product is held to 1e-5 against the fp32 oracle in
  test_gpu_raster.py, and to 1e-5 here between its culled and full-frame
  lists);
* gradients 1e-4 (the reference accumulates them with float atomics); where
  the two ops differ by more, the product must be the one within the fp32 bar
  of the float64-summed oracle.

Inputs follow the reference tests: xy uniform over the frame, scale
U(0.5, 5.5), rot U(0, 6.28), feat N(0, 1), seeded with 0xC0DA.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ATOL, ROOT, RTOL

pytestmark = pytest.mark.gpu

REF_SO = ROOT / "oracle" / "_ref" / "_C.so"


@pytest.fixture(scope="module")
def ref_op():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    if not REF_SO.exists():
        pytest.skip("reference op not built (python oracle/build_ref.py)")
    import build_ref

    return build_ref.load_built()


@pytest.fixture(scope="module")
def our_op():
    from oss_cuda import _C

    return _C


def _inputs(n, h, w, f, dev, seed=0xC0DA):
    g = torch.Generator(device=dev).manual_seed(seed)
    xy = torch.rand(n, 2, device=dev, generator=g) * torch.tensor([float(w), float(h)], device=dev)
    scale = torch.rand(n, 2, device=dev, generator=g) * 5.0 + 0.5
    rot = torch.rand(n, device=dev, generator=g) * 6.28
    feat = torch.randn(n, f, device=dev, generator=g)
    return xy.contiguous(), scale.contiguous(), rot.contiguous(), feat.contiguous()


def _near_tile_edge(xy, conic, scale, h, w, tol=1e-3):
    """Gaussians whose q = 9 box edge lies within `tol` tiles of a tile
    boundary: the only ones whose AABB may differ between two fp32
    evaluations of the same conic (the reference's cosf/sinf and approximate
    division round differently from the product's)."""
    a, b, d = conic[:, 0].double(), conic[:, 1].double(), conic[:, 2].double()
    det = a * d - b * b
    ok = det > 1e-12
    rx = torch.where(ok, torch.sqrt(9.0 * d / det.clamp_min(1e-30)), 3.0 * scale.double().max(1).values)
    ry = torch.where(ok, torch.sqrt(9.0 * a / det.clamp_min(1e-30)), 3.0 * scale.double().max(1).values)
    edges = torch.stack([(xy[:, 0].double() - rx) / 16, (xy[:, 0].double() + rx) / 16,
                         (xy[:, 1].double() - ry) / 16, (xy[:, 1].double() + ry) / 16], 1)
    return ((edges - edges.round()).abs() < tol).any(1)


def _assert_close(got, ref, atol, rtol, what):
    torch.testing.assert_close(got, ref, atol=atol, rtol=rtol, msg=lambda m: f"{what}: {m}")


@pytest.mark.parametrize("n", [1, 32, 256, 16384])
@pytest.mark.parametrize("h,w", [(128, 128), (540, 960), (1080, 1920)])
def test_preprocess_matches_reference_op(ref_op, our_op, cuda_device, n, h, w):
    xy, scale, rot, _ = _inputs(n, h, w, 1, cuda_device)
    c_r, aabb_r, pc_r = ref_op.preprocess_only(xy, scale, rot, h, w, 16)
    c_k, aabb_k, pc_k = our_op.preprocess_only(xy, scale, rot, h, w, 16)
    _assert_close(c_k, c_r, 1e-6, 1e-6, "conic")
    differ = (aabb_k != aabb_r).any(1)
    if differ.any():
        # allowed only where a box edge sits on a tile boundary to fp32 rounding
        assert bool(_near_tile_edge(xy, c_r, scale, h, w)[differ].all()), "aabb mismatch away from a tile edge"
    assert torch.equal(pc_k[~differ], pc_r[~differ]), "pair_count mismatch"


@pytest.mark.parametrize("n,h,w", [(4, 64, 64), (16, 256, 256), (64, 256, 256), (4096, 540, 960),
                                   (16384, 540, 960), (200000, 1080, 1920)])
def test_pair_construction_matches_reference_op(ref_op, our_op, cuda_device, n, h, w):
    xy, scale, rot, _ = _inputs(n, h, w, 1, cuda_device)
    if n == 200000:  # the config-2 distribution: log-scale ~ N(ln 2, 0.3)
        scale = torch.exp(torch.randn(n, 2, device=cuda_device) * 0.3 + 0.6931471805599453).contiguous()
    g_r, off_r, c_r, tot_r = ref_op.pair_construction_only(xy, scale, rot, h, w, 16)
    g_k, off_k, c_k, tot_k = our_op.pair_construction_only(xy, scale, rot, h, w, 16)
    _assert_close(c_k, c_r, 1e-6, 1e-6, "conic")
    _, aabb_r, _ = ref_op.preprocess_only(xy, scale, rot, h, w, 16)
    _, aabb_k, _ = our_op.preprocess_only(xy, scale, rot, h, w, 16)
    differ = (aabb_k != aabb_r).any(1)
    if not differ.any():
        assert int(tot_k) == int(tot_r), "total_pairs mismatch"
        assert torch.equal(g_k, g_r), "gid_sorted mismatch"
        assert torch.equal(off_k, off_r), "tile_offsets mismatch"
        return
    assert bool(_near_tile_edge(xy, c_r, scale, h, w)[differ].all()), "aabb mismatch away from a tile edge"
    # drop the boundary Gaussians from both list sets and compare the rest
    num_tiles = off_r.numel() - 1

    def strip(gid, off):
        tile = torch.repeat_interleave(torch.arange(num_tiles, device=gid.device),
                                       (off[1:] - off[:-1]).long())
        keep = ~differ[gid.long()]
        return tile[keep], gid[keep]

    t_r, s_r = strip(g_r, off_r)
    t_k, s_k = strip(g_k, off_k)
    assert torch.equal(t_k, t_r) and torch.equal(s_k, s_r), "tile lists differ beyond the boundary Gaussians"


FWD_GRID = [(n, h, w, f) for n in (0, 1, 16, 256, 4096) for (h, w) in ((32, 32), (64, 128), (270, 480), (540, 960))
            for f in (1, 3, 12, 64) if n * h * w * f <= 270_000_000]


@pytest.mark.parametrize("n,h,w,f", FWD_GRID)
def test_forward_matches_reference_op(ref_op, our_op, cuda_device, n, h, w, f):
    xy, scale, rot, feat = _inputs(n, h, w, f, cuda_device)
    out_r, g_r, off_r, c_r = ref_op.rasterize_forward(xy, scale, rot, feat, h, w, 16, True)
    out_k, _, _, c_k = our_op.rasterize_forward(xy, scale, rot, feat, h, w, 16, True)
    assert out_k.shape == out_r.shape == (f, h, w)
    _assert_close(c_k, c_r, 1e-6, 1e-6, "conic")
    _assert_close(out_k, out_r, 5e-3, 5e-3, "image (exact lists)")
    # the reference's literal full-frame lists: identical list arrays, same image
    out_f, g_f, off_f, _ = our_op.rasterize_forward(xy, scale, rot, feat, h, w, 16, True, binning="full")
    assert torch.equal(g_f, g_r) and torch.equal(off_f, off_r), "full-frame lists differ"
    _assert_close(out_f, out_r, 5e-3, 5e-3, "image (full-frame lists)")
    # exact culling changes nothing the reference's fp32 sum can see
    _assert_close(out_k, out_f, 1e-5, 1e-4, "exact vs full-frame lists")


BWD_GRID = [(n, h, w, f) for n in (1, 16, 256, 4096) for (h, w) in ((32, 32), (64, 128), (270, 480), (540, 960))
            for f in (1, 3, 12, 64) if n * h * w * f <= 270_000_000]


def _check_grad(got, ref, truth, what, bar=None):
    """Within the reference's own 1e-4 bar of the reference op.  Where not,
    the float64-summed oracle decides: each such element must be within the
    fp32 parity bar of it (`bar(t)` when given, per element), or no further
    from it than the reference op is.  Both ops sum the same fp32 terms in
    different orders (the reference with float atomics), so elements whose
    terms cancel keep a summation noise of 1e-4 and more."""
    g, r = got.detach().double().cpu(), ref.detach().double().cpu()
    near = (g - r).abs() <= 1e-4 + 1e-4 * r.abs()
    if bool(near.all()):
        return
    t = torch.as_tensor(np.asarray(truth(), np.float64))
    slack = 1e-6 * float(t.abs().max())
    eg, er = (g - t).abs(), (r - t).abs()
    meets_bar = eg <= (ATOL + slack + RTOL * t.abs() if bar is None else bar(t))
    no_worse = eg <= er + slack
    ok = near | meets_bar | no_worse
    if not bool(ok.all()):
        i = int(torch.nonzero(~ok.reshape(-1))[0])
        raise AssertionError(
            f"{what}: {int((~ok).sum())} elements differ from the reference op beyond 1e-4 and are neither within "
            f"the fp32 bar of the float64 sum nor closer to it than the reference op; first at flat index {i}: "
            f"product {float(g.reshape(-1)[i])!r}, reference {float(r.reshape(-1)[i])!r}, "
            f"float64 {float(t.reshape(-1)[i])!r}")


def _chain_rule_bars(scale, rot, d_conic):
    """Per-element fp32 bars of d_scale (N,2) and d_rot (N,): the d_conic bar
    (ATOL + 1e-6 max|d_conic| + RTOL |d_conic[g]|) carried through the chain
    rule, d_s = -2/s^3 (c^2, cs, s^2)-combination of d_conic (coefficient sum
    <= 1.5) and d_rot = (1/sx^2 - 1/sy^2) x a combination with coefficient
    sum <= 3."""
    dc = torch.as_tensor(np.asarray(d_conic, np.float64))
    s = torch.as_tensor(np.asarray(scale, np.float64)).clamp_min(1e-6)
    delta = ATOL + 1e-6 * float(dc.abs().max()) + RTOL * dc.abs().max(1).values
    amp_s = 1.5 * 2.0 / s ** 3
    diff = (1.0 / s[:, 0] ** 2 - 1.0 / s[:, 1] ** 2).abs()

    def bar_scale(t):
        return ATOL + RTOL * t.abs() + amp_s * delta[:, None]

    def bar_rot(t):
        return ATOL + RTOL * t.abs() + 3.0 * diff * delta

    return bar_scale, bar_rot


@pytest.mark.parametrize("n,h,w,f", BWD_GRID)
def test_backward_matches_reference_op(ref_op, our_op, cuda_device, n, h, w, f):
    import oracle as orc

    xy, scale, rot, feat = _inputs(n, h, w, f, cuda_device)
    _, g_r, off_r, c_r = ref_op.rasterize_forward(xy, scale, rot, feat, h, w, 16, True)
    grad = torch.randn(f, h, w, device=cuda_device, generator=torch.Generator(device=cuda_device).manual_seed(7))
    dxy_r, dc_r, df_r = ref_op.rasterize_backward(xy, scale, rot, feat, c_r, g_r, off_r, grad, h, w, 16)
    ds_r, dr_r = ref_op.conic_to_scale_rot_grad(scale, rot, dc_r)
    cpu = [t.cpu().numpy() for t in (xy, scale, rot, feat, grad)]

    # the product's backward over the reference's own lists and conic
    dxy_k, dc_k, df_k = our_op.rasterize_backward(xy, scale, rot, feat, c_r, g_r, off_r, grad, h, w, 16)
    on_ref_lists = {}

    def truth_ref_lists(i):
        if not on_ref_lists:
            on_ref_lists["v"] = orc.render_backward(cpu[0], c_r.cpu().numpy(), cpu[3], g_r.cpu().numpy(),
                                                    off_r.cpu().numpy(), cpu[4], h, w)
        return on_ref_lists["v"][i]

    for i, (name, got, ref) in enumerate((("d_xy", dxy_k, dxy_r), ("d_conic", dc_k, dc_r), ("d_feat", df_k, df_r))):
        _check_grad(got, ref, lambda i=i: truth_ref_lists(i), name + " (reference lists)")

    # the product's autograd path with its own (exact) lists
    from oss_cuda import rasterize_gaussians

    leaves = [t.detach().clone().requires_grad_(True) for t in (xy, scale, rot, feat)]
    out = rasterize_gaussians(*leaves, h, w, tile_size=16, topk_norm=True)
    out.backward(grad)
    own = {}

    def truth_own(i):
        if not own:
            own["v"] = orc.render_grads(cpu[0], cpu[1], cpu[2], cpu[3], cpu[4], h, w, mode=orc.EXACT)
        return own["v"][i]

    for name, got, ref, i in (("d_xy", leaves[0].grad, dxy_r, 0), ("d_feat", leaves[3].grad, df_r, 3)):
        _check_grad(got, ref, lambda i=i: truth_own(i), name + " (autograd)")
    # d_scale / d_rot carry the d_conic summation noise through the chain rule
    # (up to 3/s^3): their fp32 bar is the d_conic bar propagated
    bars = {}

    def bar(i):
        if not bars:
            bars["v"] = _chain_rule_bars(cpu[1], cpu[2], truth_own(5))
        return bars["v"][i - 1]

    for name, got, ref, i in (("d_scale", leaves[1].grad, ds_r, 1), ("d_rot", leaves[2].grad, dr_r, 2)):
        _check_grad(got, ref, lambda i=i: truth_own(i), name + " (autograd)", bar=lambda t, i=i: bar(i)(t))


@pytest.mark.parametrize("n", [1, 1000, 200000])
def test_conic_to_scale_rot_grad_matches_reference_op(ref_op, our_op, cuda_device, n):
    _, scale, rot, _ = _inputs(n, 64, 64, 1, cuda_device)
    d_conic = torch.randn(n, 3, device=cuda_device)
    ds_r, dr_r = ref_op.conic_to_scale_rot_grad(scale, rot, d_conic)
    ds_k, dr_k = our_op.conic_to_scale_rot_grad(scale, rot, d_conic)
    _assert_close(ds_k, ds_r, 1e-5, 1e-4, "d_scale")
    _assert_close(dr_k, dr_r, 1e-5, 1e-4, "d_rot")


@pytest.mark.parametrize("n,num_tiles", [(0, 4), (1, 1), (1000, 37), (100000, 8160)])
def test_tile_bin_counting_sort_matches_reference_op(ref_op, our_op, cuda_device, n, num_tiles):
    tile = torch.randint(0, num_tiles, (n,), device=cuda_device, dtype=torch.int32)
    gid = torch.randperm(n, device=cuda_device).to(torch.int32)
    s_r, off_r = ref_op.tile_bin_counting_sort(tile, gid, num_tiles)
    s_k, off_k = our_op.tile_bin_counting_sort(tile, gid, num_tiles)
    assert torch.equal(off_k, off_r), "offsets mismatch"
    # within a tile the reference's order is whatever its atomic cursor gave; sets must agree
    for lo, hi in zip(off_r[:-1].tolist()[:64], off_r[1:].tolist()[:64]):
        assert torch.equal(torch.sort(s_k[lo:hi]).values, torch.sort(s_r[lo:hi]).values)
    seg = torch.repeat_interleave(torch.arange(num_tiles, device=cuda_device), (off_r[1:] - off_r[:-1]).long())
    key_k = seg.long() * (n + 1) + s_k.long()
    key_r = seg.long() * (n + 1) + s_r.long()
    assert torch.equal(torch.sort(key_k).values, torch.sort(key_r).values), "per-tile sets differ"
