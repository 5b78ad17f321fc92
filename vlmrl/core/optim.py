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
from typing import Dict, Optional

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
        self.count = step
        return {"grad_norm": norm[0], "grad_sq_sum": sq[0]}

    # -------------------------------------------------------------- state access (checkpointing)
    def master_units(self) -> Dict[str, torch.Tensor]:
        return dict(self.master)

    def all_param_units(self) -> Dict[str, torch.Tensor]:
        """Every unit (frozen ones from the compute copy, trainable ones from the fp32 master)."""
        out = dict(self.params.units)
        out.update(self.master)
        return out

    def moment_units(self, which: int) -> Dict[str, torch.Tensor]:
        return dict(self.m if which == 0 else self.v)

    def load_units(self, units: Dict[str, torch.Tensor], mu=None, nu=None) -> None:
        for name, buf in self.params.units.items():
            if name in units:
                buf.copy_(units[name].to(buf.device, buf.dtype))
        for u in self.units:
            self.master[u].copy_(units[u].to(self.master[u].device, torch.float32))
            if mu is not None:
                self.m[u].copy_(mu[u].to(self.m[u].device, torch.float32))
            if nu is not None:
                self.v[u].copy_(nu[u].to(self.v[u].device, torch.float32))


def _unit_order(name: str):
    if name == "embed":
        return (0, 0)
    if name.startswith("layer"):
        return (1, int(name[5:]))
    return (2, 0)


__all__ = ["AdamWConfig", "LocalOptimizer"]
