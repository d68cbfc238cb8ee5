"""Multi-process host logic on CPU (gloo, world size 2): frame sharding, the
shared-canvas gradient all-reduce, and failure detection through a short
process-group timeout.  No GPU is touched."""
from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, outq):
    import sys

    sys.path.insert(0, str(PKG))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        import torch.distributed as dist

        from oss_b200.distributed import frame_shard, init_from_env, pack_shared_grads, reduce_shared_grads

        init_from_env(backend="gloo", timeout_s=5.0)
        if mode == "reduce":
            frames = list(frame_shard(64, rank, world))
            n_shared = 50
            packed = torch.zeros((n_shared, 9))
            for f in frames:  # per-frame gradients of the shared canvas, summed locally
                g = torch.Generator().manual_seed(f)
                grads = {"d_xy": torch.randn(60, 2, generator=g), "d_scale": torch.randn(60, 2, generator=g),
                         "d_rot": torch.randn(60, generator=g), "d_opacity": torch.randn(60, generator=g),
                         "d_rgb": torch.randn(60, 3, generator=g)}
                packed += pack_shared_grads(grads, slice(10, 60))
            reduce_shared_grads(packed)
            outq.put((rank, "ok", frames, packed))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("injected failure on rank 1 before the collective")
            t = torch.ones(4)
            dist.all_reduce(t)  # rank 1 never joins: must error out after the timeout
            outq.put((rank, "no-error", None, None))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        outq.put((rank, "error", repr(exc), traceback.format_exc()[-400:]))


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, a, b = q.get(timeout=timeout)
        out[rank] = (status, a, b)
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_frame_shard_covers_batch():
    from oss_b200.distributed import frame_shard

    for world in (1, 2, 3, 4, 8):
        got = [f for r in range(world) for f in frame_shard(64, r, world)]
        assert got == list(range(64))
    assert list(frame_shard(4, 7, 8)) == [3] and list(frame_shard(4, 6, 8)) == []
    with pytest.raises(ValueError):
        frame_shard(4, 2, 2)


def test_shared_canvas_allreduce_two_ranks():
    out = _run("reduce")
    assert out[0][0] == "ok" and out[1][0] == "ok", out
    assert out[0][1] == list(range(32)) and out[1][1] == list(range(32, 64))
    expected = torch.zeros((50, 9))
    for f in range(64):
        g = torch.Generator().manual_seed(f)
        parts = [torch.randn(60, 2, generator=g), torch.randn(60, 2, generator=g), torch.randn(60, 1, generator=g),
                 torch.randn(60, 1, generator=g), torch.randn(60, 3, generator=g)]
        expected += torch.cat(parts, dim=1)[10:60]
    for r in (0, 1):
        assert torch.allclose(out[r][2], expected, atol=1e-4)


def test_failed_rank_is_detected_by_timeout():
    out = _run("fail")
    assert out[1][0] == "error" and "injected failure" in out[1][1]
    assert out[0][0] == "error", out[0]  # the surviving rank's collective ends with an error, not a hang
