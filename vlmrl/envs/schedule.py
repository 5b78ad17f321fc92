"""Curriculum weight schedules (reference ``envs/schedule.py:15-87``).

``prepare_weight_schedule`` normalises ``{threshold: stage}`` where a stage is a
keyword (country -> only the country weight; region -> country+region;
anything else -> all three) or a mapping with ``label`` / ``weights``.  The
result is ``{threshold: {"label", "weights"}}`` sorted by threshold; an empty
or invalid schedule falls back to ``{0: full target weights}``.
"""

from __future__ import annotations

from typing import Any, Dict, Mapping, Optional

StageWeights = Dict[str, float]
DEFAULT_SCHEDULE: Dict[int, Any] = {0: "country", 1500: "region", 3000: "city"}


def weights_for_stage(stage: str, target: StageWeights) -> StageWeights:
    enabled = {"country": ("country",), "region": ("country", "region")}.get(stage.lower(), ("country", "region", "city"))
    return {k: (target[k] if k in enabled else 0.0) for k in ("country", "region", "city")}


def prepare_weight_schedule(schedule: Optional[Mapping[int, Any]], target_weights: StageWeights) -> Dict[int, Dict[str, Any]]:
    raw = dict(schedule) if schedule is not None else dict(DEFAULT_SCHEDULE)
    out: Dict[int, Dict[str, Any]] = {}
    for key, val in raw.items():
        try:
            threshold = int(key)
        except (TypeError, ValueError):
            continue
        if isinstance(val, str):
            out[threshold] = {"label": val.lower(), "weights": weights_for_stage(val, target_weights)}
        elif isinstance(val, Mapping):
            label = val.get("label")
            w = val.get("weights", val)
            if not isinstance(w, Mapping):
                continue
            out[threshold] = {
                "label": label.lower() if isinstance(label, str) else "custom",
                "weights": {"country": float(w.get("country", target_weights["country"])),
                            "region": float(w.get("region", 0.0)), "city": float(w.get("city", 0.0))},
            }
    if not out:
        out[0] = {"label": "full", "weights": dict(target_weights)}
    return dict(sorted(out.items()))


def weights_at(schedule: Mapping[int, Dict[str, Any]], step: int) -> Dict[str, Any]:
    """The entry active at ``step`` (largest threshold <= step; the first entry before it)."""
    items = sorted(schedule.items())
    active = items[0][1]
    for threshold, entry in items:
        if step >= threshold:
            active = entry
    return active


__all__ = ["prepare_weight_schedule", "weights_for_stage", "weights_at", "DEFAULT_SCHEDULE"]
