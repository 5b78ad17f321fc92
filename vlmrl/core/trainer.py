"""High-level GRPO trainer: one call = one RL iteration (rollout -> rewards -> PPO/GRPO update).

``GRPOTrainer.step()`` is the public entry point used by the CLI (``vlmrl.core.train``)
and the benchmark.  It owns the train state (AdamW), the CUDA-graph sampler,
the frozen reference model for the KL penalty, the RNG stream and the dataset
cursor (the reference's ``RollingEnv``, ``core/train.py:112-141``).  With a
process group it runs data-parallel rollouts (each rank takes its share of the
groups; rows keep global Philox ids) and an FSDP update (``vlmrl.parallel.fsdp``).

Per-phase device times (rollout, scoring+update) are measured with CUDA events
and reported with the metrics; the only host synchronisation of a step is the
token read-back that the environments need to compute rewards and the final
metric read.
"""

from __future__ import annotations

import contextlib

import time
from dataclasses import asdict
from typing import Any, Dict, Optional

import numpy as np
import torch

from vlmrl.core.kl import AdaptiveKL
from vlmrl.core.optim import AdamWConfig
from vlmrl.core.ppo import TrainerConfig, collect, update
from vlmrl.core.sampling import Generator
from vlmrl.utils.profiling import PhaseTimer, phase
from vlmrl.utils.rng import RngSeq, fold_in
from vlmrl.utils.train_state import TrainState


class GRPOTrainer:
    def __init__(self, model, tokenizer, env, cfg: TrainerConfig, adamw: AdamWConfig, *, ref_model=None,
                 seed: int = 0, master=None, eos_id: Optional[int] = None, rank: int = 0, world_size: int = 1,
                 train_state=None, tp_rollout: bool = False, tp_size: int = 0):
        self.model = model
        self.tokenizer = tokenizer
        self.env = env
        self.cfg = cfg
        self.ts = train_state if train_state is not None else TrainState.create_with_params(model, adamw, master)
        self.ref_model = ref_model
        # tp_rollout: the ranks form tensor-parallel groups of tp_size consecutive ranks (0 = all ranks).
        # Each group decodes the union of its ranks' prompt groups with 1/tp_size of each layer's weights
        # (tensor parallel over NVLink; groups are data parallel), then every rank trains on its own share
        # of the groups (FSDP over all ranks).
        self.tp = None
        self.tp_size = 1
        if tp_rollout and world_size > 1:
            from vlmrl.parallel.tp import maybe_tp_decoder, tp_subgroup

            t = int(tp_size) or int(world_size)
            group = tp_subgroup(t)
            self.tp = maybe_tp_decoder(model, group=group,
                                       max_batch=int(cfg.groups_per_batch) * max(1, int(cfg.group_size)) * t
                                       // int(world_size))
            if self.tp is not None:
                self.tp_size = t
        self.generator = Generator(model, tp=self.tp)
        self.kl_ctrl = (AdaptiveKL(cfg.kl_target, cfg.kl_adapt_rate, cfg.kl_coef_min, cfg.kl_coef_max)
                        if cfg.adaptive_kl else None)
        self.kl_coef = float(cfg.kl_coef)
        self.rng = RngSeq(seed)
        self.seed = int(seed)
        self.eos_id = eos_id if eos_id is not None else model.spec.eos_token_id
        self.rank, self.world = int(rank), int(world_size)
        self.cursor = 0
        self.iteration = 0
        self.last_collect = None
        self.last_infos: Dict[str, Any] = {}
        self.watchdog = None   # vlmrl.parallel.watchdog.Heartbeat: checked before every step

    @property
    def groups_per_rank(self) -> int:
        g = int(self.cfg.groups_per_batch)
        if g % self.world:
            raise ValueError(f"groups_per_batch={g} must be divisible by the world size {self.world}")
        return g // self.world

    def close(self) -> None:
        """Release the tensor-parallel decoder's IPC-shared buffers (collective)."""
        if self.tp is not None:
            self.tp.close()
            self.tp = None

    def state_dict(self) -> Dict[str, Any]:
        """Host state a resumed run needs besides the train state: RNG, dataset cursor, adaptive KL."""
        return {"rng": self.rng.state(), "cursor": int(self.cursor), "iteration": int(self.iteration),
                "kl_coef": float(self.kl_coef)}

    def restore_state(self, state: Optional[Dict[str, Any]]) -> None:
        if not state:
            return
        self.rng.set_state(state["rng"])
        self.cursor = int(state.get("cursor", self.cursor))
        self.iteration = int(state.get("iteration", self.iteration))
        self.kl_coef = float(state.get("kl_coef", self.kl_coef))

    def _collect(self, seed: int, G: int):
        cfg = self.cfg
        if self.tp is not None:   # the TP group rolls out its ranks' groups, then each rank keeps its share
            t = self.tp_size
            d, lr = self.rank // t, self.rank % t
            return collect(self.env, self.tokenizer, self.model, self.ts, cfg, batch_size=G * t, rng=seed,
                           eos_id=self.eos_id, generator=self.generator, task_offset=self.cursor + d * G * t,
                           row_offset=d * G * t * cfg.group_size, keep_groups=(lr * G, (lr + 1) * G))
        return collect(self.env, self.tokenizer, self.model, self.ts, cfg, batch_size=G, rng=seed, eos_id=self.eos_id,
                       generator=self.generator, task_offset=self.cursor + self.rank * G,
                       row_offset=self.rank * G * cfg.group_size)

    def rollout(self) -> Dict[str, Any]:
        """One rollout without the update: vision encode, prefill, KV-cache decode and rewards for this rank's
        groups (the inference workload; reference ``core/rollout.py`` collect + ``core/eval.py`` sampler
        benchmark).  Returns the phase times and the token counts summed over ranks."""
        if self.watchdog is not None:
            self.watchdog.check()
        timer = PhaseTimer(self.model.device)
        timer.mark("start")
        seed = self.rng.next()
        G = self.groups_per_rank
        infer = getattr(getattr(self.model, "params", None), "inference_weights", None)
        with phase("rollout"), (infer() if infer is not None else contextlib.nullcontext()):
            cr = self._collect(seed, G)
        timer.mark("rollout")
        self.cursor += G * self.world
        num_tasks = getattr(self.env, "num_tasks", -1)
        if num_tasks and num_tasks > 0:
            self.cursor %= num_tasks
        self.last_collect = cr
        eps = cr.episodes.episodes
        m: Dict[str, Any] = dict(timer.spans())
        stats = torch.tensor([float(sum(e.action_length for e in eps)), float(len(eps)),
                              float(cr.rewards.double().sum())], dtype=torch.float64, device=self.model.device)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(stats)
        m["tokens/generated"] = float(stats[0])
        m["sequences"] = float(stats[1])
        m["reward/mean"] = float(stats[2] / max(1.0, float(stats[1])))
        if self.model.device.type == "cuda":
            dec_ms = self.generator.decode_time_ms()
            if dec_ms > 0:
                m["perf/decode_tok_s"] = self.generator.last_decode_tokens / (dec_ms / 1e3)
        return m

    def step(self) -> Dict[str, Any]:
        cfg = self.cfg
        if self.watchdog is not None:
            self.watchdog.check()   # a dead peer is noticed here, before this step launches anything
        timer = PhaseTimer(self.model.device)
        timer.mark("start")
        seed = self.rng.next()
        G = self.groups_per_rank
        infer = getattr(getattr(self.model, "params", None), "inference_weights", None)
        with phase("rollout"), (infer() if infer is not None else contextlib.nullcontext()):
            cr = self._collect(seed, G)
        timer.mark("rollout")
        self.cursor += G * self.world
        num_tasks = getattr(self.env, "num_tasks", -1)
        if num_tasks and num_tasks > 0:
            self.cursor %= num_tasks
        with phase("update"):
            self.ts, m = update(self.ts, cr, cfg, ref_model=self.ref_model, kl_ctrl=self.kl_ctrl,
                                kl_coef=self.kl_coef)
        timer.mark("update")
        self.kl_coef = m.get("kl_coef", self.kl_coef)
        self.iteration += 1
        self.last_collect = cr
        self.last_infos = cr.episodes.raw_info or {}
        eps = cr.episodes.episodes
        m.update(timer.spans())
        r = cr.rewards.double()
        stats = torch.tensor([float(r.sum()), float((r * r).sum()), float(r.numel()),
                              float(sum(e.action_length for e in eps)), float(sum(len(e.full_tokens) for e in eps))],
                             dtype=torch.float64, device=self.model.device)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(stats)
        mean = stats[0] / stats[2]
        m["reward/mean"] = float(mean)
        m["reward/std"] = float((stats[1] / stats[2] - mean * mean).clamp_min(0).sqrt())
        m["tokens/generated"] = float(stats[3])
        m["tokens/total"] = float(stats[4])
        m["step"] = self.ts.step
        if self.model.device.type == "cuda":
            m["mem/allocated_gb"] = torch.cuda.memory_allocated(self.model.device) / 2 ** 30
            m["mem/peak_gb"] = torch.cuda.max_memory_allocated(self.model.device) / 2 ** 30
            dec_ms = self.generator.decode_time_ms()
            if dec_ms > 0:
                m["perf/decode_tok_s"] = self.generator.last_decode_tokens / (dec_ms / 1e3)
        if eps:
            m["sample/text"] = eps[0].generated_text[:200]
        return m


__all__ = ["GRPOTrainer"]
