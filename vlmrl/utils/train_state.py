"""Training state: parameters + AdamW state + step, saved in the reference's pickle layout.

Reference ``utils/train_state.py:16-67``: a Flax ``TrainState`` whose ``save()``
returns ``{"params", "params_ema", "opt_state", "step"}`` and whose ``step``
starts at 1.  Here the state wraps the model's parameter source and its
optimizer; ``save()`` emits the same four keys with a Flax-named NumPy params
tree and an optax-shaped ``opt_state``:

``(EmptyState(), (ScaleByAdamState(count, mu, nu), EmptyState(), EmptyState()))``

(clip_by_global_norm state, then adamw's scale_by_adam / add_decayed_weights /
scale_by_learning_rate states).  When ``optax`` is importable its NamedTuple
classes are used, so a JAX process can unpickle the file; otherwise the
same-named stand-ins below are.
"""

from __future__ import annotations

from typing import Any, Dict, NamedTuple, Optional

import numpy as np
import torch

from vlmrl.models.qwen3vl.params import all_layouts, units_to_flax, flax_to_units

try:  # pragma: no cover - optax is not part of this image
    from optax import EmptyState, ScaleByAdamState  # type: ignore
    OPTAX = True
except Exception:  # noqa: BLE001
    OPTAX = False

    class EmptyState(NamedTuple):
        """Stand-in for ``optax.EmptyState``."""

    class ScaleByAdamState(NamedTuple):
        """Stand-in for ``optax.ScaleByAdamState``."""
        count: Any
        mu: Any
        nu: Any


def _full_units(model, per_unit: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Complete a (trainable-only) unit dict with zeros so it maps onto the whole params tree."""
    out = {}
    for lay in all_layouts(model.spec):
        t = per_unit.get(lay.name)
        out[lay.name] = t if t is not None else torch.zeros(lay.numel, dtype=torch.float32)
    return out


class TrainState:
    def __init__(self, model, optimizer, step: int = 1, rng: int = 0, use_ema: bool = False):
        self.model = model
        self.optimizer = optimizer
        self.step = int(step)
        self.rng = int(rng)
        self.use_ema = bool(use_ema)
        self.params_ema: Optional[Dict[str, torch.Tensor]] = None
        if use_ema:
            self.params_ema = {u: t.detach().float().clone() for u, t in optimizer.master_units().items()}

    @classmethod
    def create_with_params(cls, model, cfg, master=None, use_ema: bool = False, rng: int = 0):
        from vlmrl.core.optim import make_optimizer

        return cls(model, make_optimizer(model.params, cfg, master=master, spec=model.spec), step=1, rng=rng,
                   use_ema=use_ema)

    def enable_ema(self) -> None:
        """Start an EMA copy of the parameters (``use_ema``) from the current master weights."""
        self.use_ema = True
        self.params_ema = {u: t.detach().float().clone() for u, t in self.optimizer.master_units().items()}

    # -------------------------------------------------------------- updates
    def apply_gradients(self) -> Dict[str, torch.Tensor]:
        metrics = self.optimizer.step(self.step)
        self.step += 1
        return metrics

    def update_ema(self, tau: float) -> None:
        if self.params_ema is None:
            return
        for u, p in self.optimizer.master_units().items():
            self.params_ema[u].mul_(tau).add_(p.float(), alpha=1 - tau)

    # -------------------------------------------------------------- (de)serialisation
    def _host_units(self, units: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return {k: v.detach().float().cpu() for k, v in units.items()}

    def save(self) -> Dict[str, Any]:
        model = self.model
        opt = self.optimizer
        master = self._host_units(opt.master_units())
        params_full = self._host_units({**{k: v for k, v in opt.all_param_units().items()}, **master})
        tree = units_to_flax(model.spec, params_full)
        ema = None
        if self.params_ema is not None:
            ema = units_to_flax(model.spec, _full_units(model, self._host_units(self.params_ema)))
        if hasattr(opt, "state_tree"):  # Adafactor: factored statistics keyed unit/leaf
            return {"params": tree, "params_ema": ema, "opt_state": {"adafactor": opt.state_tree()},
                    "step": int(self.step)}
        mu = units_to_flax(model.spec, _full_units(model, self._host_units(opt.moment_units(0))))
        nu = units_to_flax(model.spec, _full_units(model, self._host_units(opt.moment_units(1))))
        adam = ScaleByAdamState(count=np.asarray(self.step - 1, dtype=np.int32), mu=mu, nu=nu)
        inner = (adam, EmptyState(), EmptyState())
        opt_state = (EmptyState(), inner) if opt.cfg.max_grad_norm and opt.cfg.max_grad_norm > 0 else inner
        ema = None
        if self.params_ema is not None:
            ema = units_to_flax(model.spec, _full_units(model, self._host_units(self.params_ema)))
        return {"params": tree, "params_ema": ema, "opt_state": opt_state, "step": int(self.step)}

    def load(self, data: Dict[str, Any]) -> "TrainState":
        spec = self.model.spec
        units = flax_to_units(spec, data["params"])
        opt_state = data.get("opt_state")
        adam = None
        if isinstance(opt_state, dict) and "adafactor" in opt_state:
            self.optimizer.load_units(units)
            self.optimizer.load_state_tree(opt_state["adafactor"])
            self.step = int(np.asarray(data.get("step", 1)))
            return self
        if opt_state is not None:
            inner = opt_state[1] if len(opt_state) == 2 and isinstance(opt_state[1], tuple) else opt_state
            adam = inner[0]
        mu = flax_to_units(spec, adam.mu) if adam is not None else None
        nu = flax_to_units(spec, adam.nu) if adam is not None else None
        self.optimizer.load_units(units, mu, nu)
        self.step = int(np.asarray(data.get("step", 1)))
        return self


__all__ = ["TrainState", "EmptyState", "ScaleByAdamState", "OPTAX"]
