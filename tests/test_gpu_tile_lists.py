"""Tile lists by scatter + per-tile sort: bit-exact against the oracle's sorted
(tile << 32 | gid) lists in every sort tier, the device-side capacity check,
and the sync-free path captured in a CUDA graph.  Every list case runs through
both the two-call path (oss_render_prepare + oss_bin_pairs) and the one-call
path (oss_render_bin: the same kernels behind one entry point, which also
takes stacked frames).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as orc
from conftest import assert_close

pytestmark = pytest.mark.gpu

MODES = {"tight3sigma": orc.TIGHT, "exact": orc.EXACT, "exact56": orc.EXACT56}


def dev(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a), dtype=dtype).cuda().contiguous()


def host(t):
    return t.detach().cpu().numpy()


def clustered(n, h, w, seed, scale, spread=0.0):
    """n Gaussians of about `scale` px around the frame centre (+- spread px)."""
    rng = np.random.default_rng(seed)
    xy = (np.array([w, h]) / 2 + (rng.random((n, 2)) - 0.5) * 2 * spread).astype(np.float32)
    s = (scale * (0.8 + 0.4 * rng.random((n, 2)))).astype(np.float32)
    rot = (rng.random(n) * 3.14).astype(np.float32)
    return xy, s, rot


class Lists:
    """prepare + bin over the C ABI with an explicit pair capacity."""

    def __init__(self, xy, scale, rot, h, w, mode):
        from oss_cuda import _lib

        self.lib, self.chk = _lib.lib(), _lib.check
        self.n, self.h, self.w, self.mode = int(xy.shape[0]), h, w, mode
        self.tiles = ((w + 15) // 16) * ((h + 15) // 16)
        i32 = dict(device="cuda", dtype=torch.int32)
        f32 = dict(device="cuda", dtype=torch.float32)
        n = self.n
        self.xy, self.scale, self.rot = dev(xy), dev(scale), dev(rot)
        self.conic = torch.empty((n, 3), **f32)
        self.aabb = torch.empty((n, 4), **i32)
        self.pair_offset = torch.empty((n + 1,), **i32)
        self.geo = torch.empty((n, 8), **f32)
        self.total = torch.empty((1,), device="cuda", dtype=torch.int64)
        self.tile_count = torch.empty((max(1, self.lib.oss_tile_count_elems(self.tiles)),), **i32)
        self.tile_offsets = torch.empty((self.tiles + 1,), **i32)
        self.overflow = torch.full((1,), -1, **i32)
        self.prep_scratch = torch.empty((max(1, self.lib.oss_render_prepare_scratch_bytes(n)),), device="cuda",
                                        dtype=torch.uint8)
        self.pf, self.pfeat, self.popacity, self.prec = 0, None, None, None

    def pack(self, feat, opacity=None):
        """Have the preprocess also write the packed forward records."""
        self.pf, self.pfeat, self.popacity = int(feat.size(1)), feat, opacity
        self.prec = torch.empty((max(1, self.n), self.lib.oss_entry_record_floats(self.pf)), device="cuda",
                                dtype=torch.float32)

    def set_capacity(self, capacity):
        self.capacity = capacity
        self.gid = torch.full((max(1, capacity),), -7, device="cuda", dtype=torch.int32)
        nb = max(self.lib.oss_bin_pairs_scratch_bytes(self.n, capacity, self.tiles),
                 self.lib.oss_render_bin_scratch_bytes(self.n, capacity, self.tiles))
        self.scratch = torch.empty((max(1, nb),), device="cuda", dtype=torch.uint8)

    def run(self, fused=False):
        from oss_cuda import _lib

        s = torch.cuda.current_stream().cuda_stream
        if fused:
            # garbage in the outputs the one call must write
            self.pair_offset.fill_(-3)
            self.tile_offsets.fill_(-3)
            self.tile_count.fill_(12345)
            self.chk(self.lib.oss_render_bin(self.n, self.h, self.w, 1, None, self.mode, self.xy.data_ptr(),
                                             self.scale.data_ptr(), self.rot.data_ptr(), self.pf, _lib.ptr(self.pfeat),
                                             _lib.ptr(self.popacity), self.conic.data_ptr(), self.aabb.data_ptr(),
                                             self.pair_offset.data_ptr(), self.geo.data_ptr(), _lib.ptr(self.prec),
                                             self.total.data_ptr(), self.tile_count.data_ptr(),
                                             self.tile_offsets.data_ptr(), self.capacity, self.gid.data_ptr(),
                                             self.overflow.data_ptr(), self.scratch.data_ptr(), self.scratch.numel(),
                                             s), "render_bin")
            return
        self.chk(self.lib.oss_render_prepare(self.n, self.h, self.w, self.mode, self.xy.data_ptr(),
                                             self.scale.data_ptr(), self.rot.data_ptr(), self.pf,
                                             _lib.ptr(self.pfeat), _lib.ptr(self.popacity), self.conic.data_ptr(),
                                             self.aabb.data_ptr(), self.pair_offset.data_ptr(), self.geo.data_ptr(),
                                             _lib.ptr(self.prec), self.total.data_ptr(), self.tile_count.data_ptr(),
                                             self.tile_offsets.data_ptr(), self.prep_scratch.data_ptr(),
                                             self.prep_scratch.numel(), s), "prepare")
        self.chk(self.lib.oss_bin_pairs(self.n, self.h, self.w, self.mode, self.aabb.data_ptr(),
                                        self.pair_offset.data_ptr(), self.tile_count.data_ptr(),
                                        self.total.data_ptr(), self.capacity, None, None, self.gid.data_ptr(),
                                        self.tile_offsets.data_ptr(), self.overflow.data_ptr(),
                                        self.scratch.data_ptr(), self.scratch.numel(), s), "bin")


def check_lists(xy, scale, rot, h, w, mode, slack=0):
    """Both paths: lists, offsets and total against the oracle; the one-call
    path also gives the two-call path's pair offsets and per-Gaussian outputs."""
    conic, aabb, count, g_ref, o_ref = orc.lists(xy, scale, rot, h, w, MODES[mode])
    pair_ref = np.concatenate([[0], np.cumsum(count.astype(np.int64))]).astype(np.int32)
    outs = []
    for fused in (False, True):
        L = Lists(xy, scale, rot, h, w, MODES[mode])
        L.set_capacity(int(g_ref.size) + slack)
        L.run(fused=fused)
        what = "render_bin" if fused else "prepare + bin_pairs"
        assert int(L.overflow.item()) == 0, what
        assert int(L.total.item()) == g_ref.size, what
        np.testing.assert_array_equal(host(L.tile_offsets), o_ref, err_msg=what)
        np.testing.assert_array_equal(host(L.gid)[:g_ref.size], g_ref, err_msg=what)
        np.testing.assert_array_equal(host(L.pair_offset), pair_ref, err_msg=what)
        outs.append([host(t) for t in (L.conic, L.aabb, L.geo)])
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
    return o_ref


# list lengths chosen to land in each sort tier: <= 32 (warp ranks), <= 1024 (warp
# bitonic), <= 8192 (CTA bitonic), > 8192 (bitmap, one or two gid windows)
@pytest.mark.parametrize("n,h,w,scale,tier_len", [
    (30, 32, 32, 20.0, 30),
    (700, 32, 48, 30.0, 700),
    (5000, 48, 48, 40.0, 5000),
    (20000, 32, 32, 40.0, 20000),
    (300_000, 16, 16, 10.0, 300_000),
])
def test_sort_tiers_bit_exact(cuda_device, n, h, w, scale, tier_len):
    xy, s, rot = clustered(n, h, w, seed=n, scale=scale)
    o_ref = check_lists(xy, s, rot, h, w, "tight3sigma")
    assert np.diff(o_ref).max() == tier_len


@pytest.mark.parametrize("mode", ["tight3sigma", "exact", "exact56"])
def test_mixed_tiers_in_one_frame(cuda_device, mode):
    """Long lists (a dense cluster of large Gaussians) next to short ones in the
    same CTA's group of tiles."""
    rng = np.random.default_rng(3)
    h, w = 256, 384
    xy_c, s_c, rot_c = clustered(12_000, h, w, seed=5, scale=6.0, spread=40.0)
    n2 = 4000
    xy_r = (rng.random((n2, 2)) * np.array([w, h])).astype(np.float32)
    s_r = np.exp(rng.standard_normal((n2, 2)) * 0.3 + np.log(1.5)).astype(np.float32)
    rot_r = (rng.random(n2) * 3.14).astype(np.float32)
    perm = rng.permutation(12_000 + n2)
    xy = np.concatenate([xy_c, xy_r])[perm]
    s = np.concatenate([s_c, s_r])[perm]
    rot = np.concatenate([rot_c, rot_r])[perm]
    o_ref = check_lists(xy, s, rot, h, w, mode, slack=1000)
    lens = np.diff(o_ref)
    assert lens.max() > 1024 and lens.min() <= 1024


@pytest.mark.parametrize("n,h,w", [(0, 64, 64), (1, 16, 16), (5, 1, 1), (257, 37, 91), (200_000, 1080, 1920)])
def test_lists_edge_sizes(cuda_device, n, h, w):
    rng = np.random.default_rng(n)
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    s = (rng.random((n, 2)) * 3.5 + 0.5).astype(np.float32)
    rot = (rng.random(n) * 6.28).astype(np.float32)
    check_lists(xy, s, rot, h, w, "tight3sigma", slack=17)


def test_capacity_overflow_empties_lists_and_gradients(cuda_device):
    from oss_cuda import _lib

    h, w, n = 96, 160, 3000
    rng = np.random.default_rng(11)
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    s = (rng.random((n, 2)) * 3.0 + 0.5).astype(np.float32)
    rot = (rng.random(n) * 6.28).astype(np.float32)
    feat = dev(rng.random((n, 3)))
    _, _, _, g_ref, o_ref = orc.lists(xy, s, rot, h, w, orc.TIGHT)
    L = Lists(xy, s, rot, h, w, orc.TIGHT)
    L.set_capacity(int(g_ref.size) - 1)
    L.run()
    assert int(L.overflow.item()) == 1
    assert int(L.total.item()) == g_ref.size
    assert not host(L.tile_offsets).any()
    assert not host(L.pair_offset).any()
    # downstream stages stay in bounds and produce zeros
    lib, s_ = L.lib, torch.cuda.current_stream().cuda_stream
    img = torch.full((3, h, w), 5.0, device="cuda")
    _lib.check(lib.oss_render_forward(n, 3, h, w, L.geo.data_ptr(), feat.data_ptr(), None, None, L.gid.data_ptr(),
                                      L.tile_offsets.data_ptr(), img.data_ptr(), None, None, None, None, s_),
               "forward")
    assert not host(img).any()
    grad = dev(rng.standard_normal((3, h, w)))
    nb = lib.oss_render_backward_scratch_bytes(L.capacity, 3, L.tiles)
    scratch = torch.empty((nb,), device="cuda", dtype=torch.uint8)
    outs = [torch.full(sh, 9.0, device="cuda") for sh in ((n, 2), (n, 3), (n, 3))]
    _lib.check(lib.oss_render_backward(n, 3, h, w, L.geo.data_ptr(), feat.data_ptr(), None, None, None,
                                       L.aabb.data_ptr(), L.pair_offset.data_ptr(), L.capacity, L.gid.data_ptr(),
                                       L.tile_offsets.data_ptr(), None, None, grad.data_ptr(), outs[0].data_ptr(),
                                       outs[1].data_ptr(), outs[2].data_ptr(), None, None, None, scratch.data_ptr(),
                                       scratch.numel(), s_), "backward")
    for t in outs:
        assert not host(t).any()
    # the same buffers with enough room: flag cleared, lists exact
    L.set_capacity(int(g_ref.size))
    L.run()
    assert int(L.overflow.item()) == 0
    np.testing.assert_array_equal(host(L.tile_offsets), o_ref)
    np.testing.assert_array_equal(host(L.gid), g_ref)
    # the one-call path: the same overflow rule, then exact lists again
    L.set_capacity(int(g_ref.size) - 1)
    L.overflow.fill_(-1)
    L.run(fused=True)
    assert int(L.overflow.item()) == 1
    assert int(L.total.item()) == g_ref.size
    assert not host(L.tile_offsets).any()
    assert not host(L.pair_offset).any()
    L.set_capacity(int(g_ref.size))
    L.run(fused=True)
    assert int(L.overflow.item()) == 0
    np.testing.assert_array_equal(host(L.tile_offsets), o_ref)
    np.testing.assert_array_equal(host(L.gid), g_ref)


@pytest.mark.parametrize("f,dense", [(1, False), (3, False), (3, True), (5, False), (12, False), (24, False)])
def test_packed_records_and_derived_slots_bit_identical(cuda_device, f, dense):
    """The forward reading the preprocess's packed records gives the same image
    bits as the geo / feat / opacity gathers, and the backward deriving the
    pair slots gives the same gradient bits as with the forward's slots."""
    from oss_cuda import _lib

    h, w, n = 112, 176, 2500
    rng = np.random.default_rng(5 + f)
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    # dense: lists of several hundred entries (later batches staged in place)
    s = (rng.random((n, 2)) * (12.0 if dense else 3.0) + 0.5).astype(np.float32)
    rot = (rng.random(n) * 6.28).astype(np.float32)
    feat = dev(rng.standard_normal((n, f)))
    opacity = dev(rng.random(n))
    L = Lists(xy, s, rot, h, w, orc.TIGHT)
    L.pack(feat, opacity)
    L.set_capacity(int(orc.lists(xy, s, rot, h, w, orc.TIGHT)[3].size))
    L.run()
    assert int(L.overflow.item()) == 0
    lib, s_ = L.lib, torch.cuda.current_stream().cuda_stream
    rf = lib.oss_entry_record_floats(f)
    imgs, recs, slots = [], [], []
    # gathers with slots; packed records with slots; packed records without slots (the
    # persistent pipelined kernel for F <= 16)
    for packed, with_slots in ((False, True), (True, True), (True, False)):
        img = torch.empty((f, h, w), device="cuda")
        rec = torch.empty((L.capacity, rf), device="cuda")
        sl = torch.full((L.capacity,), -1, device="cuda", dtype=torch.int32)
        _lib.check(lib.oss_render_forward(n, f, h, w, L.geo.data_ptr(), feat.data_ptr(), opacity.data_ptr(),
                                          L.prec.data_ptr() if packed else None, L.gid.data_ptr(),
                                          L.tile_offsets.data_ptr(), img.data_ptr(), L.aabb.data_ptr(),
                                          L.pair_offset.data_ptr(), rec.data_ptr(),
                                          sl.data_ptr() if with_slots else None, s_), "forward")
        imgs.append(img)
        recs.append(rec)
        slots.append(sl)
    for k in (1, 2):
        assert torch.equal(imgs[0], imgs[k])
        assert torch.equal(recs[0][: L.total.item()], recs[k][: L.total.item()])
    assert torch.equal(slots[0], slots[1])
    grad = dev(rng.standard_normal((f, h, w)))
    nb = lib.oss_render_backward_scratch_bytes(L.capacity, f, L.tiles)
    grads = []
    for use_slots in (True, False):
        scratch = torch.empty((nb,), device="cuda", dtype=torch.uint8)
        outs = [torch.empty(sh, device="cuda") for sh in ((n, 2), (n, 3), (n, f), (n,), (n, 2), (n,))]
        _lib.check(lib.oss_render_backward(n, f, h, w, L.geo.data_ptr(), feat.data_ptr(), opacity.data_ptr(),
                                           L.scale.data_ptr(), L.rot.data_ptr(), L.aabb.data_ptr(),
                                           L.pair_offset.data_ptr(), L.capacity, L.gid.data_ptr(),
                                           L.tile_offsets.data_ptr(), recs[1].data_ptr(),
                                           slots[1].data_ptr() if use_slots else None, grad.data_ptr(),
                                           *[o.data_ptr() for o in outs], scratch.data_ptr(), scratch.numel(), s_),
                   "backward")
        grads.append(outs)
    for a, b in zip(*grads):
        assert torch.equal(a, b)
    # the item table built on its own (another stream) + the table-driven backward
    # write the same per-pair rows as oss_render_backward_pairs
    stride = lib.oss_pair_grad_stride(f)
    ib = lib.oss_render_backward_pairs_scratch_bytes(L.capacity, L.tiles)
    total = int(L.total.item())
    rows = []
    for split in (False, True):
        pg = torch.zeros((L.capacity, stride), device="cuda")
        items = torch.empty((ib,), device="cuda", dtype=torch.uint8)
        args = (n, f, h, w, L.geo.data_ptr(), feat.data_ptr(), opacity.data_ptr(), L.aabb.data_ptr(),
                L.pair_offset.data_ptr(), L.capacity, L.gid.data_ptr(), L.tile_offsets.data_ptr(), recs[1].data_ptr(),
                None, grad.data_ptr(), pg.data_ptr(), items.data_ptr(), ib)
        if split:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            _lib.check(lib.oss_backward_items(h, w, L.capacity, L.tile_offsets.data_ptr(), items.data_ptr(), ib,
                                              side.cuda_stream), "items")
            torch.cuda.current_stream().wait_stream(side)
            _lib.check(lib.oss_render_backward_items(*args, s_), "backward_items")
            # the table's work counter is back at zero after a launch: a second
            # backward over the same table writes every row again, identically
            first = pg[:total].clone()
            pg.zero_()
            _lib.check(lib.oss_render_backward_items(*args, s_), "backward_items again")
            assert torch.equal(first, pg[:total])
        else:
            _lib.check(lib.oss_render_backward_pairs(*args, s_), "backward_pairs")
        rows.append(pg[:total])
    assert torch.equal(rows[0], rows[1])


@pytest.mark.parametrize("fused", [False, True])
def test_sync_free_path_replays_in_cuda_graph(cuda_device, fused):
    """prepare -> bin -> forward (or render_bin -> forward) captured once,
    replayed on new Gaussians copied into the same input buffers: lists and
    image follow the new inputs."""
    from oss_cuda import _lib

    h, w, n = 128, 192, 4000
    rng = np.random.default_rng(21)

    def draw():
        xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
        s = (rng.random((n, 2)) * 3.0 + 0.5).astype(np.float32)
        rot = (rng.random(n) * 6.28).astype(np.float32)
        return xy, s, rot, rng.random((n, 3)).astype(np.float32)

    xy0, s0, r0, f0 = draw()
    L = Lists(xy0, s0, r0, h, w, orc.TIGHT)
    feat = dev(f0)
    img = torch.empty((3, h, w), device="cuda")
    L.set_capacity(4 * int(orc.lists(xy0, s0, r0, h, w, orc.TIGHT)[3].size))

    def step():
        L.run(fused=fused)
        _lib.check(L.lib.oss_render_forward(n, 3, h, w, L.geo.data_ptr(), feat.data_ptr(), None, None,
                                            L.gid.data_ptr(), L.tile_offsets.data_ptr(), img.data_ptr(), None, None,
                                            None, None, torch.cuda.current_stream().cuda_stream), "forward")

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        xy, s, rot, f = draw()
        L.xy.copy_(dev(xy))
        L.scale.copy_(dev(s))
        L.rot.copy_(dev(rot))
        feat.copy_(dev(f))
        graph.replay()
        torch.cuda.synchronize()
        c_ref, _, _, g_ref, o_ref = orc.lists(xy, s, rot, h, w, orc.TIGHT)
        assert int(L.overflow.item()) == 0
        np.testing.assert_array_equal(host(L.tile_offsets), o_ref)
        np.testing.assert_array_equal(host(L.gid)[:g_ref.size], g_ref)
        assert_close(host(img), orc.render_forward(xy, c_ref, f, g_ref, o_ref, h, w), what="graph image")
    del graph


def test_public_api_pair_capacity_mode(cuda_device):
    """rasterize_gaussians(pair_capacity=) launches without a host sync: same image
    and gradients as the default call when the capacity suffices; above it the
    lists are emptied (zero image) and the sticky flag reports it once."""
    from oss_cuda import pair_capacity_overflowed, rasterize_gaussians

    h, w, n = 80, 120, 2500
    rng = np.random.default_rng(41)
    xy = (rng.random((n, 2)) * np.array([w, h])).astype(np.float32)
    s = (rng.random((n, 2)) * 3.0 + 0.5).astype(np.float32)
    rot = (rng.random(n) * 6.28).astype(np.float32)
    feat = rng.random((n, 3)).astype(np.float32)
    grad = dev(rng.standard_normal((3, h, w)))
    total = int(orc.lists(xy, s, rot, h, w, orc.TIGHT)[3].size)
    pair_capacity_overflowed()  # clear

    def run(**kw):
        leaves = [dev(a).requires_grad_(True) for a in (xy, s, rot, feat)]
        img = rasterize_gaussians(*leaves, h, w, binning="tight3sigma", **kw)
        return [host(img)] + [host(g) for g in torch.autograd.grad(img, leaves, grad)]

    want = run()
    got = run(pair_capacity=total + 100)
    assert not pair_capacity_overflowed()
    for a, b in zip(got, want):
        np.testing.assert_array_equal(a, b)
    short = run(pair_capacity=total - 1)
    assert pair_capacity_overflowed()
    assert not pair_capacity_overflowed()  # reset by the first read
    for a in short:
        assert not a.any()


def test_item_table_lists_every_item_once_longest_first(cuda_device):
    """The backward's work-item table: every list cut into items of <= 32 entries,
    ordered by duration class (17..32 entries, 9..16, 1..8), tile order within a
    class; the item count follows the table and the work counter is cleared."""
    from oss_cuda import _lib

    lib = _lib.lib()
    ntx, nty = 8, 5
    h, w = 16 * nty - 3, 16 * ntx - 5  # ragged border tiles
    lens = [0, 1, 8, 9, 16, 17, 31, 32, 33, 40, 48, 49, 64, 65, 100, 255, 256, 257, 3, 0,
            12, 24, 7, 1000, 2, 5, 96, 97, 31, 18, 0, 0, 1, 9, 17, 33, 64, 11, 70, 5]
    assert len(lens) == ntx * nty
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    total = int(offs[-1])
    ib = lib.oss_render_backward_pairs_scratch_bytes(total, ntx * nty)
    items = torch.full((ib,), 0x5A, device="cuda", dtype=torch.uint8)
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.oss_backward_items(h, w, total, dev(offs, torch.int32).data_ptr(), items.data_ptr(), ib, s),
               "items")
    torch.cuda.synchronize()
    raw = host(items)
    max_items = ntx * nty + (total + 31) // 32
    off = ((max_items * 16 + 255) // 256) * 256
    count, counter = raw[off:off + 8].view(np.int32)
    table = raw[:max_items * 16].view(np.int32).reshape(max_items, 4)[:count]

    want = {0: [], 1: [], 2: []}
    for t, n in enumerate(lens):
        for i in range(n // 32):
            want[0].append((t, int(offs[t]) + 32 * i, 32))
        rest = n % 32
        if rest:
            want[0 if rest > 16 else (1 if rest > 8 else 2)].append((t, int(offs[t]) + n - rest, rest))
    expect = want[0] + want[1] + want[2]
    assert count == len(expect)
    assert counter == 0
    assert [tuple(map(int, r[:3])) for r in table] == expect
