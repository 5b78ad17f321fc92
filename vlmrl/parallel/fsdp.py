"""FSDP engine: sharded parameter units, per-unit gradient reduce-scatter and sharded AdamW.

Counterpart of reference ``utils/sharding.py:23-48`` (defined there but never
wired in): here FSDP is the training path for N > 1 GPUs.

Layout: every parameter unit (``vlmrl.models.qwen3vl.params``) is padded to a
multiple of ``128 * world`` elements and split into ``world`` contiguous
shards.  Rank r keeps shard r of: the bf16 compute copy, the fp32 master, the
AdamW moments and the fp32 gradient.

* ``get(unit)`` all-gathers the bf16 unit on first use and keeps it until the
  next optimizer step (the forward's gathered weights serve the backward too:
  with 180 GB of HBM a replicated bf16 copy of a 4-8B model is cheap, so only
  the fp32 optimizer state — 16 bytes/param — is sharded).
* ``grad(unit)`` hands the executor a full-size fp32 accumulator;
  ``grad_done(unit)`` reduce-scatters it (sum) into this rank's gradient shard
  on a side stream, overlapped with the backward of the next unit.
* ``FSDPOptimizer.step`` computes the global gradient norm (shard sums
  all-reduced), clips, runs the AdamW kernel on the shards (which also writes
  the bf16 shard) and invalidates the gathered copies.

Collectives go through NCCL (``vlmrl.parallel.dist``); the NVLink peer-memory
kernels in ``vlmrl.parallel.symm`` replace them where a fused path exists.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Sequence

import torch
import torch.distributed as dist

from vlmrl import ops
from vlmrl.core.optim import AdamWConfig, _unit_order
from vlmrl.models.qwen3vl.params import UnitLayout
from vlmrl.parallel.dist import all_gather_into, all_reduce_, reduce_scatter_into


class FSDPParams:
    def __init__(self, layouts: Sequence[UnitLayout], full_units: Dict[str, torch.Tensor], *, group=None,
                 dtype=torch.bfloat16, trainable: Optional[Iterable[str]] = None, replicate: Iterable[str] = ()):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dtype = dtype
        self.layouts = {l.name: l for l in layouts}
        self.trainable = set(trainable) if trainable is not None else {l.name for l in layouts if l.trainable}
        self.replicated: Dict[str, torch.Tensor] = {}
        self.shards: Dict[str, torch.Tensor] = {}
        self.padded: Dict[str, int] = {}
        self.gathered: Dict[str, torch.Tensor] = {}
        self.grads_full: Dict[str, torch.Tensor] = {}
        self.grad_shards: Dict[str, torch.Tensor] = {}
        self._pending: List = []
        self.device = next(iter(full_units.values())).device
        self.comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        rep = set(replicate)
        for name, lay in self.layouts.items():
            full = full_units[name]
            if name in rep or name not in self.trainable:
                self.replicated[name] = full.to(dtype).contiguous()
                continue
            P = lay.padded_numel(self.world)
            n = P // self.world
            self.padded[name] = P
            buf = torch.zeros(P, dtype=dtype, device=self.device)
            buf[:lay.numel].copy_(full[:lay.numel])
            self.shards[name] = buf[self.rank * n:(self.rank + 1) * n].clone()
            self.grad_shards[name] = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.units = self.replicated  # frozen units, for code that wants a plain dict

    # ---------------------------------------------------------------- ParamSource protocol
    def get(self, name: str) -> torch.Tensor:
        if name in self.replicated:
            return self.replicated[name]
        buf = self.gathered.get(name)
        if buf is None:
            buf = torch.empty(self.padded[name], dtype=self.dtype, device=self.device)
            all_gather_into(buf, self.shards[name], group=self.group)
            self.gathered[name] = buf
        return buf[:self.layouts[name].numel]

    def release(self, name: str) -> None:
        pass

    def grad(self, name: str) -> Optional[torch.Tensor]:
        if name not in self.trainable or name in self.replicated:
            return None
        g = self.grads_full.get(name)
        if g is None:
            g = torch.zeros(self.padded[name], dtype=torch.float32, device=self.device)
            self.grads_full[name] = g
        return g[:self.layouts[name].numel]

    def grad_done(self, name: str) -> None:
        g = self.grads_full.pop(name, None)
        if g is None:
            return
        out = torch.empty_like(self.grad_shards[name])
        if self.comm_stream is not None:
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                reduce_scatter_into(out, g, group=self.group)
                self.grad_shards[name].add_(out)
            g.record_stream(self.comm_stream)
            out.record_stream(self.comm_stream)
        else:
            reduce_scatter_into(out, g, group=self.group)
            self.grad_shards[name].add_(out)

    def sync_grads(self) -> None:
        if self.comm_stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)

    def invalidate(self) -> None:
        self.gathered.clear()

    def zero_grads(self) -> None:
        for g in self.grad_shards.values():
            g.zero_()

    def full_unit(self, name: str) -> torch.Tensor:
        """Gathered unit (collective: every rank must call it)."""
        return self.get(name)


class FSDPOptimizer:
    """AdamW over the local shards; the global gradient norm is an all-reduce of shard sums."""

    def __init__(self, params: FSDPParams, cfg: AdamWConfig):
        self.params = params
        self.cfg = cfg
        self.units = sorted(params.shards, key=_unit_order)
        self.master = {u: params.shards[u].float().clone() for u in self.units}
        self.m = {u: torch.zeros_like(self.master[u]) for u in self.units}
        self.v = {u: torch.zeros_like(self.master[u]) for u in self.units}

    def step(self, step: int) -> Dict[str, torch.Tensor]:
        p, c = self.params, self.cfg
        p.sync_grads()
        sq = torch.zeros(1, dtype=torch.float32, device=p.device)
        for u in self.units:
            ops.sq_norm(p.grad_shards[u], out=sq)
        all_reduce_(sq, group=p.group)
        norm = sq.sqrt()
        scale = torch.clamp(c.max_grad_norm / (norm + 1e-12), max=1.0) if c.max_grad_norm and c.max_grad_norm > 0 \
            else torch.ones_like(norm)
        for u in self.units:
            ops.adamw_(self.master[u], p.grad_shards[u], self.m[u], self.v[u], lr=c.lr, beta1=c.beta1, beta2=c.beta2,
                       eps=c.eps, weight_decay=c.weight_decay, step=step, grad_scale=scale, p_half=p.shards[u])
            p.grad_shards[u].zero_()
        p.invalidate()
        return {"grad_norm": norm[0], "grad_sq_sum": sq[0]}

    # ---------------------------------------------------------------- checkpointing (collectives)
    def _gather(self, shards: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        p = self.params
        out = {}
        for u in self.units:
            full = torch.empty(p.padded[u], dtype=shards[u].dtype, device=p.device)
            all_gather_into(full, shards[u], group=p.group)
            out[u] = full[:p.layouts[u].numel]
        return out

    def master_units(self) -> Dict[str, torch.Tensor]:
        return self._gather(self.master)

    def all_param_units(self) -> Dict[str, torch.Tensor]:
        out = dict(self.params.replicated)
        out.update(self.master_units())
        return out

    def moment_units(self, which: int) -> Dict[str, torch.Tensor]:
        return self._gather(self.m if which == 0 else self.v)

    def load_units(self, units: Dict[str, torch.Tensor], mu=None, nu=None) -> None:
        p = self.params
        for name, buf in p.replicated.items():
            if name in units:
                buf.copy_(units[name].to(buf.device, buf.dtype))
        for u in self.units:
            n = p.padded[u] // p.world
            sl = slice(p.rank * n, (p.rank + 1) * n)

            def shard_of(t):
                full = torch.zeros(p.padded[u], dtype=torch.float32, device=p.device)
                full[:p.layouts[u].numel].copy_(t[:p.layouts[u].numel].to(p.device, torch.float32))
                return full[sl]

            self.master[u].copy_(shard_of(units[u]))
            p.shards[u].copy_(self.master[u].to(p.shards[u].dtype))
            if mu is not None:
                self.m[u].copy_(shard_of(mu[u]))
            if nu is not None:
                self.v[u].copy_(shard_of(nu[u]))
        p.invalidate()


def build_fsdp_models(spec, adamw: AdamWConfig, *, seed: int = 0, device=None, group=None, dtype=torch.bfloat16,
                      units: Optional[Dict[str, torch.Tensor]] = None):
    """-> (policy model on FSDP params, frozen replicated reference model, TrainState).

    ``units`` (full parameter units, e.g. loaded from a checkpoint) replace the seeded random init.
    """
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.models.qwen3vl.params import all_layouts, init_params, text_layouts
    from vlmrl.utils.train_state import TrainState

    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if units is None:
        units = init_params(spec, seed=seed, dtype=dtype, device=device)
    else:
        units = {k: v.to(device, dtype) for k, v in units.items()}
    ref = Qwen3VLModel(spec, units={k: v for k, v in units.items() if k != "visual"}, device=device, dtype=dtype)
    fp = FSDPParams(all_layouts(spec), units, group=group, dtype=dtype,
                    trainable=[l.name for l in text_layouts(spec)], replicate=["visual"])
    del units
    model = Qwen3VLModel(spec, params=fp, device=device, dtype=dtype)
    if not isinstance(adamw, AdamWConfig):
        raise NotImplementedError("the FSDP engine shards AdamW state only (factored Adafactor statistics need "
                                  "whole rows); use optimizer=adamw or a single process")
    ts = TrainState(model, FSDPOptimizer(fp, adamw))
    return model, ref, ts


__all__ = ["FSDPParams", "FSDPOptimizer", "build_fsdp_models"]
