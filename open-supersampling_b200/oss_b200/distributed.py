"""Multi-GPU plumbing for batched rendering (one process per GPU).

Frames and their canvases are independent (the reference keeps each rank's
canvas unsynchronised, oss/sr/v6/model.py:39-42), so a batch is split into
contiguous frame shards with no data-path collective.  The one exchange is the
shared-canvas gradient: each rank sums the gradients of a canvas shared by all
frames over its own frames, then one all-reduce (NCCL over NVLink on GPUs,
gloo on CPU) makes every rank hold the total.  Process groups get a short
timeout so that a rank that fails or never joins ends the others' next
collective with an error instead of a hang.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def frame_shard(total: int, rank: int, world: int) -> range:
    """Contiguous frames [total*rank/world, total*(rank+1)/world) of this rank."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world: {rank}/{world}")
    return range(total * rank // world, total * (rank + 1) // world)


def init_from_env(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Join the process group described by RANK/WORLD_SIZE/MASTER_ADDR/MASTER_PORT
    (torchrun).  Returns (rank, world, local_rank); world 1 needs no group."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kwargs)
    return rank, world, local


SHARED_GRAD_FIELDS = (("d_xy", 2), ("d_scale", 2), ("d_rot", 1), ("d_opacity", 1), ("d_rgb", 3))


def pack_shared_grads(grads: dict, sl: slice) -> torch.Tensor:
    """(n, 9) rows of the shared Gaussians' gradients in a fixed field order."""
    cols = []
    for name, width in SHARED_GRAD_FIELDS:
        g = grads[name][sl]
        cols.append(g.reshape(g.shape[0], width))
    return torch.cat(cols, dim=1)


def reduce_shared_grads(packed: torch.Tensor) -> torch.Tensor:
    """Sum the packed shared-canvas gradients over all ranks, in place."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(packed, op=dist.ReduceOp.SUM)
    return packed
