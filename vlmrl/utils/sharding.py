"""DP / FSDP sharding plans and data helpers over ``torch.distributed`` (reference ``utils/sharding.py:11-104``).

The reference defines a 1-D device mesh with two plans (never wired into its
trainer): ``dp`` replicates the train state, ``fsdp`` shards every parameter
larger than 4 MiB on its first axis divisible by the device count.  Here one
process drives one GPU, so a "plan" is a per-leaf decision that the FSDP engine
(``vlmrl.parallel.fsdp``) realises with padded flat shards, and the data
helpers slice the global batch for this rank:

* ``create_sharding(kind, shapes)`` -> ``(param_plan, replicate, data_spec, shard_data)``;
* ``shard_data(*xs)`` keeps rows ``[r*n/W, (r+1)*n/W)`` of every array whose
  leading dimension divides by the world size and leaves the others whole
  (the reference's replication fallback);
* ``host_gather`` all-gathers a tensor or picklable object across ranks;
* ``get_local_slice`` is the rank's slice of a global batch;
* ``get_memory_usage`` reports GiB allocated on this rank's GPU.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

MIN_SIZE_TO_SHARD_MB = 4


def _world() -> Tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


@dataclass(frozen=True)
class LeafPlan:
    """Sharded axis of one parameter leaf (None = replicated)."""
    axis: Optional[int]


def shard_axis(shape: Sequence[int], itemsize: int, world: int) -> Optional[int]:
    """First axis divisible by ``world`` for leaves above 4 MiB, else None (reference rule)."""
    if int(np.prod(shape)) * itemsize <= MIN_SIZE_TO_SHARD_MB * (2 ** 20):
        return None
    for i, s in enumerate(shape):
        if s % world == 0:
            return i
    return None


def create_sharding(shard_type: str, train_state_shape: Optional[Dict[str, Any]] = None, world: Optional[int] = None):
    """-> (param_plan, replicate_plan, data_plan, shard_data); ``train_state_shape`` maps leaf name -> array/shape."""
    rank, w = _world()
    w = int(world or w)
    replicate = LeafPlan(None)
    data_plan = LeafPlan(0)
    if shard_type == "dp":
        plan: Any = replicate
    elif shard_type == "fsdp":
        plan = {}
        for name, leaf in (train_state_shape or {}).items():
            shape = tuple(getattr(leaf, "shape", leaf))
            itemsize = getattr(getattr(leaf, "dtype", None), "itemsize", 4) or 4
            if isinstance(leaf, torch.Tensor):
                itemsize = leaf.element_size()
            plan[name] = LeafPlan(shard_axis(shape, int(itemsize), w))
    else:
        raise ValueError(f"unknown shard_type {shard_type!r} (dp or fsdp)")

    def shard_data(*args):
        def one(x):
            if x is None or not hasattr(x, "shape") or len(x.shape) == 0 or x.shape[0] % w:
                return x
            n = x.shape[0] // w
            return x[rank * n:(rank + 1) * n]

        return one(args[0]) if len(args) == 1 else tuple(one(a) for a in args)

    return plan, replicate, data_plan, shard_data


def host_gather(x):
    """Concatenate ``x`` from every rank (tensor: along dim 0; other objects: a list)."""
    rank, w = _world()
    if w == 1:
        return x
    if isinstance(x, torch.Tensor):
        parts = [torch.empty_like(x) for _ in range(w)]
        dist.all_gather(parts, x.contiguous())
        return torch.cat(parts)
    out = [None] * w
    dist.all_gather_object(out, x)
    return out


def get_local_slice(x, world: Optional[int] = None, rank: Optional[int] = None):
    """This rank's contiguous slice of a global batch along dim 0."""
    r, w = _world()
    r = r if rank is None else int(rank)
    w = w if world is None else int(world)
    n = x.shape[0] // w
    return x[r * n:(r + 1) * n]


def get_memory_usage() -> float:
    """GiB currently allocated by this process on its GPU (0 without CUDA)."""
    if not torch.cuda.is_available():
        return 0.0
    return torch.cuda.memory_allocated() / (1024 ** 3)


__all__ = ["LeafPlan", "shard_axis", "create_sharding", "host_gather", "get_local_slice", "get_memory_usage"]
