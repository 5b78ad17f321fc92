"""FSDP engine: sharded parameter units, per-unit gradient reduce-scatter and sharded AdamW.

Counterpart of reference ``utils/sharding.py:23-48`` (defined there but never
wired in): here FSDP is the training path for N > 1 GPUs.

Layout: every parameter unit (``vlmrl.models.qwen3vl.params``) is padded to a
multiple of ``128 * world`` elements and split into ``world`` contiguous
shards.  Rank r keeps shard r of: the bf16 compute copy, the fp32 master, the
AdamW moments and the fp32 gradient.  The bf16 unit is kept gathered (with
180 GB of HBM a replicated bf16 copy of a 4-8B model is cheap, so only the
fp32 optimizer state — 16 bytes/param — is sharded).

Communication (``comm``):

* ``p2p`` (default with NCCL ranks on one node): gathered bf16 units and the
  full-size fp32 gradients live in IPC-shared buffers mapped by every rank
  (``vlmrl.parallel.symm``).  ``grad_done(unit)`` launches the peer-pull
  reduce-scatter kernel on a side stream (overlapped with the backward of the
  next unit); ``FSDPOptimizer.step`` all-reduces the squared norm (one float),
  then one fused kernel per unit applies AdamW to the shard and stores the bf16
  result into every rank's gathered unit; a bounded device-side wait publishes
  them.  No NCCL all-gather or reduce-scatter runs in a step.
* ``nccl`` (also gloo on CPU): NCCL/gloo reduce-scatter per unit and an
  all-gather of each stale unit on first use after a step — the baseline.

Sharded parameters (``shard_params=True`` with ``p2p``; ZeRO-3 style, for
models whose bf16 copy should not stay resident next to the activations):
the decoder-layer units keep only their bf16 shard, in an IPC-shared buffer.
The training forward and backward read the four weight matrices of a layer
through ``ops.ShardedWeight``: the GEMM that consumes a matrix copies its
rows from every rank's shard into a local work buffer inside the kernel,
chunk by chunk, while its MMAs run (the all-gather fused into the GEMM);
the small leaves (norm weights, biases) come from one ``unit_gather``
kernel per layer.  Two work buffers alternate between consecutive layers.
Rollout runs inside ``inference_weights()``, which gathers whole units into
a temporary copy.  The optimizer writes the new bf16 shard in place and a
device-side barrier publishes it before the next gather reads it.
"""

from __future__ import annotations

import contextlib
import os
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from vlmrl import ops
from vlmrl.ops._ext import ext
from vlmrl.core.optim import AdamWConfig, _unit_order, frozen_decay
from vlmrl.models.qwen3vl.params import UnitLayout
from vlmrl.parallel.dist import all_gather_into, all_reduce_, reduce_scatter_into


_CHECK_COLLECTIVES = os.environ.get("VLMRL_CHECK_COLLECTIVES", "0") == "1"

# matrices of a decoder-layer unit that sharded-parameter mode gathers inside their GEMMs
GATHERED_LEAVES = ("qkv_w", "o_w", "gu_w", "down_w")


def _small_ranges(layout: UnitLayout, skip: Sequence[str]) -> List[Tuple[int, int]]:
    """Byte ranges of a unit's leaves outside ``skip`` (16-byte rounded, neighbours merged)."""
    out: List[Tuple[int, int]] = []
    for prm in layout.params:
        if prm.name in skip:
            continue
        a = layout.offsets[prm.name] * 2
        b = -(-(layout.offsets[prm.name] + prm.numel) * 2 // 16) * 16
        if out and a <= -(-out[-1][1] // 256) * 256:
            out[-1] = (out[-1][0], max(out[-1][1], b))
        else:
            out.append((a, b))
    return out


class FSDPParams:
    """Sharded parameter source for the executor (``get``/``grad``/``grad_done`` protocol).

    ``comm="p2p"`` (default with NCCL on one node): gathered bf16 units and
    full-size fp32 gradients live in IPC-shared buffers (``SymmetricBuffer``);
    ``grad_done`` launches the peer-pull reduce-scatter kernel and the
    optimizer's fused AdamW kernel stores the new bf16 shard into every rank's
    gathered copy, so no NCCL all-gather or reduce-scatter runs in a step.
    ``comm="nccl"`` (and gloo on CPU): the same protocol over NCCL/gloo
    collectives, the baseline the fused path is measured against.  Both keep
    the gathered buffers at fixed addresses, so CUDA graphs that captured them
    stay valid across optimizer steps.
    """

    def __init__(self, layouts: Sequence[UnitLayout], full_units: Dict[str, torch.Tensor], *, group=None,
                 dtype=torch.bfloat16, trainable: Optional[Iterable[str]] = None, replicate: Iterable[str] = (),
                 comm: Optional[str] = None, shard_params: Optional[bool] = None):
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
        self.fresh: Dict[str, bool] = {}
        self.grads_full: Dict[str, torch.Tensor] = {}
        self.grad_shards: Dict[str, torch.Tensor] = {}
        self.device = next(iter(full_units.values())).device
        self.comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        if comm is None:
            comm = os.environ.get("VLMRL_FSDP_COMM", "p2p")
        if comm == "p2p":
            from vlmrl.parallel.symm import p2p_supported

            if self.device.type != "cuda" or self.world > 8 or not p2p_supported(group):
                comm = "nccl"
        self.comm = comm
        if shard_params is None:
            shard_params = os.environ.get("VLMRL_FSDP_SHARD_PARAMS", "0") == "1"
        self.shard_params = bool(shard_params) and comm == "p2p"
        self.sharded: List[str] = []
        self._infer: Optional[Dict[str, torch.Tensor]] = None
        self.graph_epoch = 0          # changes whenever inference weights move (captured graphs are stale)
        rep = set(replicate)
        sharded = []
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
            sharded.append(name)
        self.order = sorted(sharded, key=_unit_order)
        self.slot = {u: i for i, u in enumerate(self.order)}
        if self.comm == "p2p":
            self._init_p2p()
        else:
            for u in self.order:
                self.gathered[u] = torch.empty(self.padded[u], dtype=dtype, device=self.device)
                self.fresh[u] = False
        self.units = self.replicated  # frozen units, for code that wants a plain dict
        self.version = 0              # bumped by every optimizer step (consumers re-slice derived copies)

    # ---------------------------------------------------------------- peer-memory setup
    def _init_p2p(self) -> None:
        from vlmrl.parallel.symm import SymmetricBuffer

        W = self.world
        self.g_off: Dict[str, int] = {}
        self.p_off: Dict[str, int] = {}
        self.s_off: Dict[str, int] = {}
        self.sharded = [u for u in self.order if self.shard_params and u.startswith("layer")]
        self.sharded_set = set(self.sharded)
        go = po = so = 0
        for u in self.order:
            self.g_off[u] = go
            go += self.padded[u] * 4
            if u in self.sharded_set:
                self.s_off[u] = so
                so += self.padded[u] // W * 2
            else:
                self.p_off[u] = po
                po += self.padded[u] * 2
        self.sym_grad = SymmetricBuffer(go, self.group, self.device)
        self.sym_param = SymmetricBuffer(max(po, 256), self.group, self.device)
        self.sym_shard = None
        if self.sharded:
            self.sym_shard = SymmetricBuffer(so, self.group, self.device)
            big = max(self.padded[u] for u in self.sharded)
            self.work = [torch.empty(big, dtype=self.dtype, device=self.device) for _ in range(2)]
            self.g_flags = torch.zeros(8192, dtype=torch.int32, device=self.device)
            self.g_ctr = torch.zeros(2, dtype=torch.int32, device=self.device)
            self.ranges = {u: _small_ranges(self.layouts[u], GATHERED_LEAVES) for u in self.sharded}
        self.n_slots = len(self.order) + 2          # one per unit (reduce-scatter), push, barrier
        self.sym_sig = SymmetricBuffer(self.n_slots * W * 8, self.group, self.device)
        self.push_slot, self.barrier_slot = len(self.order), len(self.order) + 1
        self.rs_epoch = [0] * len(self.order)
        self.push_target = 0
        self.barrier_epoch = 0
        self.grad_live: Dict[str, bool] = {}
        self.reduced: Dict[str, bool] = {u: False for u in self.order}
        for u in self.order:
            self.grads_full[u] = self.sym_grad.view(self.g_off[u], (self.padded[u],), torch.float32)
            self.grad_live[u] = False
            self.fresh[u] = True
            if u in self.sharded_set:
                view = self.sym_shard.view(self.s_off[u], (self.padded[u] // W,), self.dtype)
                view.copy_(self.shards[u])
                self.shards[u] = view       # the optimizer writes the gather source in place
                continue
            self.gathered[u] = self.sym_param.view(self.p_off[u], (self.padded[u],), self.dtype)
            all_gather_into(self.gathered[u], self.shards[u], group=self.group)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def verify_signals(self) -> None:
        """Debug check of the peer-memory protocol (``VLMRL_CHECK_COLLECTIVES=1`` runs it after every step).

        After a step's device-side wait, every peer's counters in this rank's signal pad must equal the
        values this rank expects exactly: a smaller value is a lost signal, a larger one a peer that ran
        ahead of the protocol (a race).  Reads the pad to the host (synchronises).
        """
        if self.comm != "p2p":
            return
        W = self.world
        pad = self.sym_sig.view(0, (self.n_slots, W), torch.int64).cpu()
        bad = []
        for i, u in enumerate(self.order):
            for q in range(W):
                if q != self.rank and int(pad[i, q]) != self.rs_epoch[i]:
                    bad.append(f"reduce-scatter {u}: rank {q} at {int(pad[i, q])}, expected {self.rs_epoch[i]}")
        for q in range(W):
            if q != self.rank and int(pad[self.push_slot, q]) != self.push_target:
                bad.append(f"parameter push: rank {q} at {int(pad[self.push_slot, q])}, expected {self.push_target}")
        if bad:
            raise RuntimeError("peer-memory collective counters out of step: " + "; ".join(bad[:6]))

    def close(self) -> None:
        """Release the IPC-shared buffers (collective)."""
        if self.comm == "p2p":
            for b in (self.sym_grad, self.sym_param, self.sym_sig, self.sym_shard):
                if b is not None:
                    b.close()
            self.gathered.clear()
            self.grads_full.clear()
            self.comm = "closed"

    # ---------------------------------------------------------------- sharded parameters
    def _shard_srcs(self, name: str) -> Tuple[List[int], int]:
        return [ptr + self.s_off[name] for ptr in self.sym_shard.ptrs], self.padded[name] // self.world * 2

    def _gather_whole(self, name: str) -> torch.Tensor:
        full = torch.empty(self.padded[name], dtype=self.dtype, device=self.device)
        srcs, sb = self._shard_srcs(name)
        ops.unit_gather(srcs, full.data_ptr(), sb, [(0, self.padded[name] * 2)])
        return full

    def views(self, name: str, layout: UnitLayout) -> Optional[Dict[str, object]]:
        """Executor hook: the leaves of a sharded unit, its matrices as ``ops.ShardedWeight`` (gathered by the
        GEMMs that read them).  None for every other unit (the executor then slices ``get(name)``)."""
        if name not in getattr(self, "sharded_set", ()):
            return None
        if self._infer is not None:
            return layout.views(self._infer[name])
        buf = self.work[int(name[len("layer"):]) % 2]
        srcs, sb = self._shard_srcs(name)
        base = buf.data_ptr()
        ops.unit_gather(srcs, base, sb, self.ranges[name])
        v: Dict[str, object] = dict(layout.views(buf))
        for k in GATHERED_LEAVES:
            if k in v:
                v[k] = ops.ShardedWeight(v[k], srcs, base, sb, self.g_flags, self.g_ctr)
        return v

    @contextlib.contextmanager
    def inference_weights(self):
        """Whole copies of the sharded units for rollout (decode graphs need plain weight tensors); freed on
        exit.  A no-op without sharded parameters."""
        if not self.sharded or self._infer is not None:
            yield
            return
        self._infer = {u: self._gather_whole(u) for u in self.sharded}
        self.graph_epoch += 1
        try:
            yield
        finally:
            self._infer = None
            self.graph_epoch += 1

    # ---------------------------------------------------------------- ParamSource protocol
    def get(self, name: str) -> torch.Tensor:
        if name in self.replicated:
            return self.replicated[name]
        if name in getattr(self, "sharded_set", ()):
            full = self._infer[name] if self._infer is not None else self._gather_whole(name)
            return full[:self.layouts[name].numel]
        buf = self.gathered[name]
        if not self.fresh[name]:
            all_gather_into(buf, self.shards[name], group=self.group)
            self.fresh[name] = True
        return buf[:self.layouts[name].numel]

    def release(self, name: str) -> None:
        pass

    def grad(self, name: str) -> Optional[torch.Tensor]:
        if name not in self.trainable or name in self.replicated:
            return None
        if self.comm == "p2p":
            g = self.grads_full[name]
            if not self.grad_live[name]:
                if self.reduced[name]:
                    # a peer may still be pulling from this buffer (no optimizer step since the last
                    # reduce-scatter): wait for every rank's reduce-scatters before overwriting it
                    self.sync_grads()
                    self.barrier_epoch += 1
                    ext().peer_barrier(self.sym_sig.ptrs, self.barrier_slot, self.barrier_epoch, self.rank,
                                       self.sym_sig.dev_index)
                    for u in self.reduced:
                        self.reduced[u] = False
                g.zero_()
                self.grad_live[name] = True
            return g[:self.layouts[name].numel]
        g = self.grads_full.get(name)
        if g is None:
            g = torch.zeros(self.padded[name], dtype=torch.float32, device=self.device)
            self.grads_full[name] = g
        return g[:self.layouts[name].numel]

    def grad_done(self, name: str) -> None:
        if self.comm == "p2p":
            if not self.grad_live.get(name):
                return
            self.grad_live[name] = False
            self.reduced[name] = True
            i = self.slot[name]
            self.rs_epoch[i] += 1
            n = self.padded[name] // self.world
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                ext().rs_pull(self.sym_grad.ptrs, self.g_off[name], self.rank * n, self.grad_shards[name], True,
                                  self.sym_sig.ptrs, i, self.rs_epoch[i], self.rank, 0)
            return
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
        """The shards changed (optimizer step or load): gathered copies are stale until re-gathered."""
        if self.comm != "p2p":
            for u in self.fresh:
                self.fresh[u] = False

    def zero_grads(self) -> None:
        for g in self.grad_shards.values():
            g.zero_()

    def full_unit(self, name: str) -> torch.Tensor:
        """Gathered unit (collective: every rank must call it)."""
        return self.get(name)

    def regather(self) -> None:
        """Refill every gathered buffer from the shards (collective; used after loading a checkpoint)."""
        for u in self.order:
            if u in self.gathered:
                all_gather_into(self.gathered[u], self.shards[u], group=self.group)
        if self.sharded:    # peers read the reloaded shards directly: publish them
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.fresh[u] = True


class FSDPOptimizer:
    """AdamW over the local shards; the global gradient norm is an all-reduce of shard sums.

    With peer-memory communication the AdamW kernel also performs the
    parameter all-gather (``adamw_push``) and one bounded device-side wait
    (``peer_wait``) publishes the new parameters before the next forward.
    """

    def __init__(self, params: FSDPParams, cfg: AdamWConfig):
        self.params = params
        self.cfg = cfg
        self.units = sorted(params.shards, key=_unit_order)
        self.master = {u: params.shards[u].float().clone() for u in self.units}
        self.m = {u: torch.zeros_like(self.master[u]) for u in self.units}
        self.v = {u: torch.zeros_like(self.master[u]) for u in self.units}
        # replicated frozen units decay identically on every rank (no communication)
        self.frozen = frozen_decay(params.replicated, params.trainable, cfg)

    def step(self, step: int) -> Dict[str, torch.Tensor]:
        p, c = self.params, self.cfg
        if self.frozen is not None:
            self.frozen.step(c.lr, c.weight_decay)
        p.sync_grads()
        sq = torch.zeros(1, dtype=torch.float32, device=p.device)
        for u in self.units:
            ops.sq_norm(p.grad_shards[u], out=sq)
        all_reduce_(sq, group=p.group)
        norm = sq.sqrt()
        scale = torch.clamp(c.max_grad_norm / (norm + 1e-12), max=1.0) if c.max_grad_norm and c.max_grad_norm > 0 \
            else torch.ones_like(norm)
        if p.comm == "p2p":
            W = p.world
            for u in self.units:
                if u in p.sharded_set:
                    # sharded parameters: the new bf16 shard is written in place; peers gather it later
                    ops.adamw_(self.master[u], p.grad_shards[u], self.m[u], self.v[u], lr=c.lr, beta1=c.beta1,
                               beta2=c.beta2, eps=c.eps, weight_decay=c.weight_decay, step=step, grad_scale=scale,
                               p_half=p.shards[u])
                    p.grad_shards[u].zero_()
                    continue
                n = p.padded[u] // W
                grid = ext().adamw_push(self.master[u], p.grad_shards[u], self.m[u], self.v[u], p.sym_param.ptrs,
                                            p.p_off[u] + p.rank * n * 2, scale, c.lr, c.beta1, c.beta2, c.eps,
                                            c.weight_decay, step, p.sym_sig.ptrs, p.push_slot, p.rank)
                p.push_target += int(grid)
                p.shards[u].copy_(self.master[u])
                p.grad_shards[u].zero_()
            ext().peer_wait(p.sym_sig.local, p.push_slot, p.push_target, p.rank, W, p.sym_sig.dev_index)
            if p.sharded:
                # every rank's shards are updated before any rank's next gather reads them
                p.barrier_epoch += 1
                ext().peer_barrier(p.sym_sig.ptrs, p.barrier_slot, p.barrier_epoch, p.rank, p.sym_sig.dev_index)
            if _CHECK_COLLECTIVES:
                ops.check_errors(p.sym_sig.dev_index)
                p.verify_signals()
            for u in p.reduced:
                p.reduced[u] = False
        else:
            for u in self.units:
                ops.adamw_(self.master[u], p.grad_shards[u], self.m[u], self.v[u], lr=c.lr, beta1=c.beta1,
                           beta2=c.beta2, eps=c.eps, weight_decay=c.weight_decay, step=step, grad_scale=scale,
                           p_half=p.shards[u])
                p.grad_shards[u].zero_()
            p.invalidate()
        p.version += 1
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
        if self.frozen is not None:
            out.update(self.frozen.master)
        out.update(self.master_units())
        return out

    def moment_units(self, which: int) -> Dict[str, torch.Tensor]:
        return self._gather(self.m if which == 0 else self.v)

    def load_units(self, units: Dict[str, torch.Tensor], mu=None, nu=None) -> None:
        p = self.params
        for name, buf in p.replicated.items():
            if name in units:
                buf.copy_(units[name].to(buf.device, buf.dtype))
                if self.frozen is not None and name in self.frozen.master:
                    self.frozen.master[name].copy_(units[name].to(buf.device, torch.float32))
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
        p.version += 1
        if p.comm == "p2p":
            p.regather()


def build_fsdp_models(spec, adamw: AdamWConfig, *, seed: int = 0, device=None, group=None, dtype=torch.bfloat16,
                      units: Optional[Dict[str, torch.Tensor]] = None, shard_params: Optional[bool] = None):
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
                    trainable=[l.name for l in text_layouts(spec)], replicate=["visual"], shard_params=shard_params)
    del units
    model = Qwen3VLModel(spec, params=fp, device=device, dtype=dtype)
    if not isinstance(adamw, AdamWConfig):
        raise NotImplementedError("the FSDP engine shards AdamW state only (factored Adafactor statistics need "
                                  "whole rows); use optimizer=adamw or a single process")
    ts = TrainState(model, FSDPOptimizer(fp, adamw))
    return model, ref, ts


__all__ = ["FSDPParams", "FSDPOptimizer", "build_fsdp_models"]
