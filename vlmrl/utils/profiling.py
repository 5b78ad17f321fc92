"""Tracing hooks: NVTX ranges per phase and CUDA-event phase timers.

``phase(name)`` opens an NVTX range (visible in Nsight Systems and in
``ncu --nvtx`` filters) around a phase of the RL step — rollout, prefill,
decode, reward, scoring, update, optimizer — and is free when CUDA is absent.
``PhaseTimer`` records CUDA events at phase boundaries on the current stream
and reports device milliseconds per phase without synchronising until read;
``max_over_ranks`` turns a local time into the job's (slowest rank) time.

No reference counterpart beyond the eval CLI's wall-clock timing
(``core/eval.py:65-71,146-166``).
"""

from __future__ import annotations

import contextlib
import time
from typing import Dict, List, Tuple

import torch


@contextlib.contextmanager
def phase(name: str):
    on = torch.cuda.is_available()
    if on:
        torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        if on:
            torch.cuda.nvtx.range_pop()


class PhaseTimer:
    """``mark(name)`` closes the previous phase and opens ``name``; ``spans()`` -> {time/<name>_ms}."""

    def __init__(self, device=None):
        dev = torch.device(device) if device is not None else None
        self.cuda = torch.cuda.is_available() and (dev is None or dev.type == "cuda")
        self.marks: List[Tuple[str, object]] = []

    def mark(self, name: str) -> None:
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.marks.append((name, e))
        else:
            self.marks.append((name, time.perf_counter()))

    def spans(self) -> Dict[str, float]:
        out: Dict[str, float] = {}
        if self.cuda and self.marks:
            self.marks[-1][1].synchronize()
        for (_, ta), (b, tb) in zip(self.marks, self.marks[1:]):
            out[f"time/{b}_ms"] = ta.elapsed_time(tb) if self.cuda else (tb - ta) * 1e3
        return out


def max_over_ranks(value: float) -> float:
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


__all__ = ["phase", "PhaseTimer", "max_over_ranks"]
