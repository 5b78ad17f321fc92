"""AdamW with global-norm clipping over flat parameter units (optax ``chain(clip_by_global_norm, adamw)``).

Reference optimizer: ``core/train.py:211-234`` — ``clip_by_global_norm(max)``
then ``adamw(lr, b1=0.9, b2=0.999, eps=1e-8, weight_decay)``; the decoupled
decay is applied to every trainable leaf (here: every trainable unit).

Each trainable unit has an fp32 master copy, first/second moments and an fp32
gradient accumulator; the compute copy (bf16) is rewritten by the AdamW kernel
in the same pass.  The clip scale ``min(1, max_norm / ||g||)`` is computed on
the device and read by the kernel from device memory, so the step never
synchronises with the host.  ``grad_norm`` is the true L2 norm (the reference
logs the squared norm; that value is reported as ``grad_sq_sum``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import torch

from vlmrl import ops


@dataclass
class AdamWConfig:
    lr: float = 1e-6
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 1e-2
    max_grad_norm: float = 1.0
    # the reference's optax chain decays every leaf, the gradient-free vision tower included (reference
    # core/train.py:225-228); on: frozen units drift by (1 - lr * weight_decay) per step as there
    decay_frozen: bool = False


class FrozenDecay:
    """Decoupled weight decay of gradient-free units: ``p <- p * (1 - lr * wd)`` every optimizer step.

    AdamW with a zero gradient leaves both moments at zero, so its step on such a leaf is the decay term
    alone.  The product is kept in an fp32 copy (per-step factors such as 1 - 1e-8 are below bf16
    resolution) and written back to the compute copy after each step.
    """

    def __init__(self, units: Dict[str, torch.Tensor]):
        self.units = units
        self.master = {u: t.detach().float().clone() for u, t in units.items()}

    def step(self, lr: float, weight_decay: float) -> None:
        f = 1.0 - float(lr) * float(weight_decay)
        for u, m in self.master.items():
            m.mul_(f)
            self.units[u].copy_(m)

    def reseed(self, names=None) -> None:
        """Take the compute copies as the new starting point (after a checkpoint load)."""
        for u in (self.master if names is None else [n for n in names if n in self.master]):
            self.master[u].copy_(self.units[u])


def frozen_decay(units: Dict[str, torch.Tensor], trainable, cfg) -> Optional[FrozenDecay]:
    if not getattr(cfg, "decay_frozen", False) or not getattr(cfg, "weight_decay", 0.0):
        return None
    frozen = {u: t for u, t in units.items() if u not in set(trainable)}
    return FrozenDecay(frozen) if frozen else None


class LocalOptimizer:
    """Optimizer state for a ``LocalParams`` source (all units resident on one device)."""

    def __init__(self, params, cfg: AdamWConfig, master: Optional[Dict[str, torch.Tensor]] = None):
        self.params = params
        self.cfg = cfg
        self.units = sorted(params.trainable, key=_unit_order)
        self.master: Dict[str, torch.Tensor] = {}
        self.m: Dict[str, torch.Tensor] = {}
        self.v: Dict[str, torch.Tensor] = {}
        for u in self.units:
            src = master[u] if master is not None and u in master else params.units[u]
            dev = params.units[u].device
            self.master[u] = src.detach().to(dev, torch.float32).clone()
            self.m[u] = torch.zeros_like(self.master[u])
            self.v[u] = torch.zeros_like(self.master[u])
            params.grad(u)
        self.count = 0
        self.frozen = frozen_decay(params.units, params.trainable, cfg)

    def grad_sq_sum(self) -> torch.Tensor:
        dev = self.master[self.units[0]].device
        acc = torch.zeros(1, dtype=torch.float32, device=dev)
        for u in self.units:
            ops.sq_norm(self.params.grads[u], out=acc)
        return acc

    def step(self, step: int) -> Dict[str, torch.Tensor]:
        """One AdamW update with bias correction at ``step`` (1-based); zeroes the gradients."""
        c = self.cfg
        sq = self.grad_sq_sum()
        norm = sq.sqrt()
        if c.max_grad_norm and c.max_grad_norm > 0:
            scale = torch.clamp(c.max_grad_norm / (norm + 1e-12), max=1.0)
        else:
            scale = torch.ones_like(norm)
        for u in self.units:
            ops.adamw_(self.master[u], self.params.grads[u], self.m[u], self.v[u], lr=c.lr, beta1=c.beta1,
                       beta2=c.beta2, eps=c.eps, weight_decay=c.weight_decay, step=step, grad_scale=scale,
                       p_half=self.params.units[u])
            self.params.grads[u].zero_()
        if self.frozen is not None:
            self.frozen.step(c.lr, c.weight_decay)
        self.count = step
        return {"grad_norm": norm[0], "grad_sq_sum": sq[0]}

    # -------------------------------------------------------------- state access (checkpointing)
    def master_units(self) -> Dict[str, torch.Tensor]:
        return dict(self.master)

    def all_param_units(self) -> Dict[str, torch.Tensor]:
        """Every unit (frozen ones from the compute copy or their decay copy, trainable ones from the fp32 master)."""
        out = dict(self.params.units)
        if self.frozen is not None:
            out.update(self.frozen.master)
        out.update(self.master)
        return out

    def moment_units(self, which: int) -> Dict[str, torch.Tensor]:
        return dict(self.m if which == 0 else self.v)

    def load_units(self, units: Dict[str, torch.Tensor], mu=None, nu=None) -> None:
        for name, buf in self.params.units.items():
            if name in units:
                buf.copy_(units[name].to(buf.device, buf.dtype))
        if self.frozen is not None:
            for name in units:
                if name in self.frozen.master:
                    self.frozen.master[name].copy_(units[name].to(self.frozen.master[name].device, torch.float32))
        for u in self.units:
            self.master[u].copy_(units[u].to(self.master[u].device, torch.float32))
            if mu is not None:
                self.m[u].copy_(mu[u].to(self.m[u].device, torch.float32))
            if nu is not None:
                self.v[u].copy_(nu[u].to(self.v[u].device, torch.float32))


@dataclass
class AdafactorConfig:
    """``optax.adafactor`` as the reference configures it (``core/train.py:217-223``), after global-norm clipping."""
    lr: float = 1e-6
    weight_decay: float = 1e-2
    max_grad_norm: float = 1.0
    min_dim_size_to_factor: int = 32
    decay_rate: float = 0.8
    decay_offset: int = 0
    clipping_threshold: float = 1.0
    min_param_scale: float = 1e-3
    eps: float = 1e-30


def leaf_views(spec, unit: str, flat: torch.Tensor) -> List[Tuple[str, torch.Tensor]]:
    """The Flax leaves of one text unit as views of its flat buffer.

    The fused ``qkv_w``/``qkv_b`` rows split into the q, k and v leaves; the
    row-interleaved ``gu_w`` splits into gate (even rows) and up (odd rows).
    Per-leaf statistics (factored second moments, block RMS) therefore match
    an optimizer that runs on the reference's parameter tree.
    """
    from vlmrl.models.qwen3vl.params import all_layouts

    lay = {l.name: l for l in all_layouts(spec)}[unit]
    t = spec.text
    nq, nkv = t.num_attention_heads * t.head_dim, t.num_key_value_heads * t.head_dim
    out: List[Tuple[str, torch.Tensor]] = []
    for name, v in lay.views(flat).items():
        if unit.startswith("layer") and name in ("qkv_w", "qkv_b"):
            out += [(name + ".q", v[:nq]), (name + ".k", v[nq:nq + nkv]), (name + ".v", v[nq + nkv:])]
        elif unit.startswith("layer") and name == "gu_w":
            out += [("gu_w.gate", v[0::2]), ("gu_w.up", v[1::2])]
        else:
            out.append((name, v))
    return out


def _factored_dims(shape, min_dim: int):
    """(reduce-for-column, reduce-for-row) axes: the two largest dims, or None (Shazeer & Stern 2018, sec. 3)."""
    if len(shape) < 2:
        return None
    order = sorted(range(len(shape)), key=lambda i: shape[i])
    if shape[order[-2]] < min_dim:
        return None
    return order[-2], order[-1]


def _rms(x: torch.Tensor) -> torch.Tensor:
    return x.float().pow(2).mean().sqrt()


class LocalAdafactor:
    """Adafactor (factored second moments, update clipping, relative step scale, decoupled decay).

    Follows Shazeer & Stern, "Adafactor: Adaptive Learning Rates with Sublinear
    Memory Cost" (2018) in the form ``optax.adafactor`` composes it: factored
    RMS scaling with decay ``1 - (t+1)^-0.8``, update clipping at block RMS 1,
    learning-rate scale, multiplication by ``max(rms(param), 1e-3)``, then
    ``+ weight_decay * param`` and a negative step.  Preceded by global-norm
    clipping of the raw gradient, as the reference chains it.  Runs as torch
    ops over each leaf (a secondary optimizer; the AdamW path has its own kernel).
    """

    def __init__(self, params, cfg: AdafactorConfig, master: Optional[Dict[str, torch.Tensor]] = None, spec=None):
        self.params = params
        self.cfg = cfg
        self.spec = spec
        self.units = sorted(params.trainable, key=_unit_order)
        self.master: Dict[str, torch.Tensor] = {}
        self.state: Dict[str, Dict[str, Tuple[torch.Tensor, ...]]] = {}
        for u in self.units:
            src = master[u] if master is not None and u in master else params.units[u]
            dev = params.units[u].device
            self.master[u] = src.detach().to(dev, torch.float32).clone()
            params.grad(u)
            st = {}
            for name, v in leaf_views(spec, u, self.master[u]):
                fd = _factored_dims(tuple(v.shape), cfg.min_dim_size_to_factor)
                if fd is None:
                    st[name] = (torch.zeros_like(v),)
                else:
                    d1, d0 = fd
                    st[name] = (v.new_zeros([s for i, s in enumerate(v.shape) if i != d0]),
                                v.new_zeros([s for i, s in enumerate(v.shape) if i != d1]))
            self.state[u] = st
        self.count = 0

    def step(self, step: int) -> Dict[str, torch.Tensor]:
        c = self.cfg
        dev = self.master[self.units[0]].device
        sq = torch.zeros(1, dtype=torch.float32, device=dev)
        for u in self.units:
            ops.sq_norm(self.params.grads[u], out=sq)
        norm = sq.sqrt()
        gscale = torch.clamp(c.max_grad_norm / (norm + 1e-12), max=1.0) if c.max_grad_norm and c.max_grad_norm > 0 \
            else torch.ones_like(norm)
        t = float(self.count - c.decay_offset + 1)
        decay = 1.0 - t ** (-c.decay_rate)
        for u in self.units:
            grads = dict(leaf_views(self.spec, u, self.params.grads[u]))
            for name, p in leaf_views(self.spec, u, self.master[u]):
                g = grads[name] * gscale
                g2 = g * g + c.eps
                st = self.state[u][name]
                fd = _factored_dims(tuple(p.shape), c.min_dim_size_to_factor)
                if fd is None:
                    (v,) = st
                    v.mul_(decay).add_(g2, alpha=1.0 - decay)
                    upd = g * v.rsqrt()
                else:
                    d1, d0 = fd
                    vr, vc = st
                    vr.mul_(decay).add_(g2.mean(d0), alpha=1.0 - decay)
                    vc.mul_(decay).add_(g2.mean(d1), alpha=1.0 - decay)
                    red = d1 - 1 if d1 > d0 else d1
                    row = (vr / vr.mean(red, keepdim=True)).rsqrt()
                    upd = g * row.unsqueeze(d0) * vc.rsqrt().unsqueeze(d1)
                upd = upd / torch.clamp(_rms(upd) / c.clipping_threshold, min=1.0)
                upd = upd * c.lr * torch.clamp(_rms(p), min=c.min_param_scale)
                if c.weight_decay and c.weight_decay > 0:
                    upd = upd + c.weight_decay * p
                p.sub_(upd)
            self.params.units[u].copy_(self.master[u].to(self.params.units[u].dtype))
            self.params.grads[u].zero_()
        self.count += 1
        return {"grad_norm": norm[0], "grad_sq_sum": sq[0]}

    def master_units(self) -> Dict[str, torch.Tensor]:
        return dict(self.master)

    def all_param_units(self) -> Dict[str, torch.Tensor]:
        out = dict(self.params.units)
        out.update(self.master)
        return out

    def state_tree(self) -> Dict[str, Any]:
        """Factored statistics keyed ``unit/leaf`` (host copies) plus the step count."""
        out: Dict[str, Any] = {"count": int(self.count)}
        for u, st in self.state.items():
            for name, tensors in st.items():
                out[f"{u}/{name}"] = tuple(x.detach().cpu().numpy() for x in tensors)
        return out

    def load_state_tree(self, tree: Dict[str, Any]) -> None:
        self.count = int(tree.get("count", 0))
        for u, st in self.state.items():
            for name, tensors in st.items():
                for dst, src in zip(tensors, tree[f"{u}/{name}"]):
                    dst.copy_(torch.as_tensor(src))

    def load_units(self, units: Dict[str, torch.Tensor], mu=None, nu=None) -> None:
        for name, buf in self.params.units.items():
            if name in units:
                buf.copy_(units[name].to(buf.device, buf.dtype))
        for u in self.units:
            self.master[u].copy_(units[u].to(self.master[u].device, torch.float32))


def make_optimizer(params, cfg, master: Optional[Dict[str, torch.Tensor]] = None, spec=None):
    """LocalOptimizer for an AdamWConfig, LocalAdafactor for an AdafactorConfig."""
    if isinstance(cfg, AdafactorConfig):
        if spec is None:
            raise ValueError("Adafactor needs the model spec to split units into parameter leaves")
        return LocalAdafactor(params, cfg, master=master, spec=spec)
    return LocalOptimizer(params, cfg, master=master)


def _unit_order(name: str):
    if name == "embed":
        return (0, 0)
    if name.startswith("layer"):
        return (1, int(name[5:]))
    return (2, 0)


__all__ = ["AdamWConfig", "AdafactorConfig", "LocalOptimizer", "LocalAdafactor", "make_optimizer", "leaf_views"]
