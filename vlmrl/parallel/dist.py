"""Process-group plumbing: init from torchrun-style env vars, rank helpers, collectives that also run on gloo.

``init_from_env`` reads ``RANK`` / ``WORLD_SIZE`` / ``LOCAL_RANK`` /
``MASTER_ADDR`` / ``MASTER_PORT``, picks NCCL on GPUs and gloo on CPU, and
gives the group a finite timeout so ranks that wait on a dead peer fail with an
error instead of hanging.  ``all_gather_into`` / ``reduce_scatter_into`` use the
tensor collectives on NCCL and an all-reduce fallback on gloo (which lacks
reduce-scatter), so the FSDP engine is testable on CPU ranks.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    backend: str = "none"

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def info() -> DistInfo:
    if dist.is_available() and dist.is_initialized():
        return DistInfo(dist.get_rank(), dist.get_world_size(), int(os.environ.get("LOCAL_RANK", dist.get_rank())),
                        dist.get_backend())
    return DistInfo(local_rank=int(os.environ.get("LOCAL_RANK", "0")))


def init_from_env(timeout_s: float = 600.0, backend: Optional[str] = None) -> DistInfo:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1 or (dist.is_initialized()):
        return info()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return info()


def _is_gloo(group=None) -> bool:
    return dist.get_backend(group) == "gloo"


def all_gather_into(out: torch.Tensor, shard: torch.Tensor, group=None, async_op: bool = False):
    """out[r*n:(r+1)*n] = shard of rank r."""
    if _is_gloo(group):
        parts = list(out.chunk(dist.get_world_size(group)))
        dist.all_gather(parts, shard.contiguous(), group=group)
        return None
    return dist.all_gather_into_tensor(out, shard, group=group, async_op=async_op)


def reduce_scatter_into(out: torch.Tensor, full: torch.Tensor, group=None, async_op: bool = False):
    """out = sum over ranks of full[r*n:(r+1)*n] for this rank r."""
    if _is_gloo(group):
        tmp = full.clone()
        dist.all_reduce(tmp, group=group)
        r = dist.get_rank(group)
        out.copy_(tmp.chunk(dist.get_world_size(group))[r])
        return None
    return dist.reduce_scatter_tensor(out, full, group=group, async_op=async_op)


def all_reduce_(t: torch.Tensor, op=dist.ReduceOp.SUM, group=None) -> torch.Tensor:
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=op, group=group)
    return t


def barrier(group=None) -> None:
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.barrier(group=group)


__all__ = ["DistInfo", "info", "init_from_env", "all_gather_into", "reduce_scatter_into", "all_reduce_", "barrier"]
