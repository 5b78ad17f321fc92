"""Metric logging: W&B when requested, JSONL on disk by default.

Reference ``utils/wandb.py:62-194`` drives W&B directly.  Here ``MetricLogger``
writes one JSON line per ``log`` call (offline-safe) and mirrors to W&B only
when ``mode`` is ``online``/``offline`` and the package imports.
``summarize_env_metrics`` reproduces the reference's env-metric aggregation:
means of the tracked keys, last ``stage_idx``, within-{25,100,500} km rates,
distance p50/p90 and the 1:2:3-weighted coordinate-quality score.
"""

from __future__ import annotations

import json
import os
import time
from typing import Any, Dict, Iterable, List, Optional

import numpy as np

ENV_METRIC_SUMMARIES = {
    "env/stage_acc": "mean", "env/city_correct": "mean", "env/distance_km": "mean",
    "env/within_25km": "mean", "env/within_100km": "mean", "env/within_500km": "mean",
    "env/distance_p50": "mean", "env/distance_p90": "mean", "env/format_ok": "mean",
    "env/parsed_field_count": "mean", "env/coord_quality_score": "mean",
    "env/final_reward": "mean", "env/stage_idx": "last",
}
_MEAN_KEYS = ("stage_acc", "city_correct", "distance_km", "format_ok", "parsed_field_count", "final_reward")
_COORD_KEYS = ("has_coords", "coords_in_range", "coords_within_tolerance")
_ALLOWED = set(_MEAN_KEYS) | {"stage_idx"} | set(_COORD_KEYS)


def _numbers(value: Any) -> List[float]:
    if isinstance(value, dict):
        return [x for v in value.values() for x in _numbers(v)]
    if isinstance(value, (list, tuple, set)):
        return [x for v in value for x in _numbers(v)]
    if hasattr(value, "shape"):
        arr = np.asarray(value, dtype=np.float32).reshape(-1)
        return arr.tolist()
    if isinstance(value, (bool, int, float, np.number)):
        return [float(value)]
    return []


def summarize_env_metrics(env_infos: Dict[str, Iterable[Any]]) -> Dict[str, float]:
    out: Dict[str, float] = {}
    arrays: Dict[str, np.ndarray] = {}
    for key, raw in env_infos.items():
        if key not in _ALLOWED:
            continue
        vals = _numbers(raw)
        if not vals:
            continue
        arr = np.asarray(vals, dtype=np.float32)
        arrays[key] = arr
        if key == "stage_idx":
            out["env/stage_idx"] = float(arr[-1])
        else:
            out[f"env/{key}"] = float(arr.mean())
    dist = arrays.get("distance_km")
    if dist is not None and dist.size:
        for t in (25, 100, 500):
            out[f"env/within_{t}km"] = float(np.mean(dist <= t))
        for p in (50, 90):
            out[f"env/distance_p{p}"] = float(np.percentile(dist, p))
    comps = [arrays[k].mean() for k in _COORD_KEYS if k in arrays]
    if comps:
        w = np.arange(1, len(comps) + 1, dtype=np.float32)
        out["env/coord_quality_score"] = float(np.dot(np.asarray(comps, dtype=np.float32), w) / w.sum())
    return out


class MetricLogger:
    """JSONL metric sink with optional W&B mirroring (rank 0 only)."""

    def __init__(self, path: Optional[str] = None, *, mode: str = "disabled", project: str = "vlmrl",
                 name: Optional[str] = None, group: Optional[str] = None, entity: Optional[str] = None,
                 config: Optional[Dict[str, Any]] = None, rank: int = 0):
        self.rank = rank
        self.path = path
        self._fh = None
        self._wandb = None
        if rank != 0:
            return
        if path:
            os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
            self._fh = open(path, "a", encoding="utf-8")
        if mode in ("online", "offline"):
            try:
                import wandb  # noqa: F401

                self._wandb = wandb.init(project=project, name=name, group=group, entity=entity or None,
                                         mode=mode, config=config or {})
                define_env_metrics()
            except Exception:  # W&B is best-effort, as in the reference trainer
                self._wandb = None

    def log(self, metrics: Dict[str, Any], step: int) -> None:
        if self.rank != 0:
            return
        row = {}
        for k, v in metrics.items():
            if isinstance(v, (int, float, str, bool)) or v is None:
                row[k] = v
            elif hasattr(v, "item"):
                row[k] = v.item()
        row.update(step=int(step), time=time.time())  # the explicit step wins over a metric named "step"
        if self._fh:
            self._fh.write(json.dumps(row) + "\n")
            self._fh.flush()
        if self._wandb is not None:
            try:
                self._wandb.log({**row, "global_step": int(step)})
            except Exception:
                pass

    def close(self) -> None:
        if self._fh:
            self._fh.close()
            self._fh = None
        if self._wandb is not None:
            try:
                self._wandb.finish()
            except Exception:
                pass


def define_env_metrics() -> None:
    try:
        import wandb

        wandb.define_metric("global_step")
        wandb.define_metric("*", step_metric="global_step")
        for metric, summary in ENV_METRIC_SUMMARIES.items():
            wandb.define_metric(metric, summary=summary)
    except Exception:
        pass


def setup_wandb(hyperparam_dict: Dict[str, Any], entity=None, project="vlmrl", group=None, name=None,
                offline: bool = False, **_: Any):
    """Reference-compatible entry point returning a ``MetricLogger`` bound to W&B."""
    return MetricLogger(None, mode="offline" if offline else "online", project=project, name=name,
                        group=group, entity=entity, config=hyperparam_dict)


__all__ = ["MetricLogger", "summarize_env_metrics", "define_env_metrics", "setup_wandb", "ENV_METRIC_SUMMARIES"]
