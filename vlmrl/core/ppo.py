"""PPO / GRPO learner: ``TrainerConfig``, ``collect`` and ``update`` (reference ``core/ppo.py:28-254``).

``collect`` samples ``groups_per_batch x group_size`` episodes in one batched
rollout and builds one packed batch per minibatch.  ``update`` runs, for every
epoch and minibatch: the policy forward with activations saved, the per-token
loss (``vlmrl.core.grpo.ppo_loss``), the explicit backward and one AdamW step.

Old log-probs (``old_logprob_source``):
* ``"policy"`` (default) — the policy's own scoring pass before any update, so
  the first minibatch starts at ratio 1 (the first minibatch reuses its own
  training forward; later minibatches are scored up front);
* ``"sampler"`` — the sampler's log-probs (the reference's behaviour, which
  uses the tempered/top-k masked distribution).
KL to the frozen reference policy uses the reference model's log-probs on the
same tokens, computed once per iteration.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from vlmrl.core.batching import pack_groups, pack_sequences
from vlmrl.core.grpo import group_advantages, ppo_loss, token_advantages
from vlmrl.core.kl import AdaptiveKL
from vlmrl.core.minibatch import minibatch_indices
from vlmrl.core.rollout import EpisodeBatch, collect_episodes
from vlmrl.core.types import Rollout, SamplingConfig
from vlmrl.models.qwen3vl.model import PackedBatch
from vlmrl.utils.profiling import phase


@dataclass
class TrainerConfig:
    temperature: float = 0.7
    top_p: Optional[float] = 0.9
    top_k: Optional[int] = 1024
    max_new_tokens: int = 64
    max_sequence_length: int = 2048
    clip_epsilon: float = 0.2
    entropy_coef: float = 0.0
    kl_coef: float = 0.0
    adaptive_kl: bool = False
    kl_target: float = 0.02
    kl_adapt_rate: float = 1.5
    kl_coef_min: float = 1e-5
    kl_coef_max: float = 0.5
    ppo_minibatch: int = 64
    ppo_epochs: int = 1
    n_minibatches: int = 0
    groups_per_batch: int = 16
    group_size: int = 1
    kl_ref_coef: float = 0.0
    adv_norm: str = "group"
    old_logprob_source: str = "policy"
    # rollouts start like the reference's sampler (last prompt token decoded twice); for parity runs only
    compat_refeed_last_token: bool = False
    share_prompt: bool = True
    vlm_min_pixels: int = -1
    vlm_max_pixels: int = -1


@dataclass
class MiniBatch:
    batch: PackedBatch
    seq_index: np.ndarray          # episode indices in this minibatch
    counts: np.ndarray             # scored tokens per sequence
    adv_tok: torch.Tensor          # [M]
    sampler_lp: torch.Tensor       # [M]
    old_lp: Optional[torch.Tensor] = None
    ref_lp: Optional[torch.Tensor] = None


@dataclass
class CollectResult:
    episodes: EpisodeBatch
    rewards: torch.Tensor
    advantages: torch.Tensor
    minibatches: List[MiniBatch] = field(default_factory=list)
    rollout: Optional[Rollout] = None


def sampling_config(cfg: TrainerConfig, eos_id: Optional[int], pad_id: int = 0) -> SamplingConfig:
    return SamplingConfig(temperature=cfg.temperature, top_p=cfg.top_p, top_k=cfg.top_k, eos_id=eos_id,
                          pad_id=pad_id, max_new_tokens=cfg.max_new_tokens,
                          compat_refeed_last_token=bool(getattr(cfg, "compat_refeed_last_token", False)))


def _minibatch_count(cfg: TrainerConfig, n: int) -> int:
    if cfg.n_minibatches and cfg.n_minibatches > 0:
        return int(cfg.n_minibatches)
    return max(1, n // max(1, int(cfg.ppo_minibatch)))


def _groups_of(idx: np.ndarray, eps, group_size: int):
    """Split minibatch episode indices into whole groups (consecutive members), or None if they are not."""
    if group_size <= 1 or len(idx) % group_size:
        return None
    out = []
    for g in range(0, len(idx), group_size):
        members = idx[g:g + group_size]
        gid = eps[members[0]].group_id
        if np.any(np.diff(members) != 1) or any(eps[i].group_id != gid for i in members):
            return None
        out.append(members)
    return out


def build_minibatches(model, eb: EpisodeBatch, adv_seq: torch.Tensor, n_minibatches: int,
                      max_sequence_length: Optional[int] = None, share_prompt: bool = True) -> List[MiniBatch]:
    """Packed minibatches; with ``share_prompt`` each group's prompt is computed once (``pack_groups``)."""
    eps = eb.episodes
    merge = model.spec.vision.spatial_merge_size
    # vision rows per episode (episodes are stored contiguously in eb.vision)
    counts_img = [sum(int(t) * (int(h) // merge) * (int(w) // merge) for t, h, w in ep.grids) for ep in eps]
    starts = np.concatenate([[0], np.cumsum(counts_img)])
    out: List[MiniBatch] = []
    for idx in minibatch_indices(len(eps), n_minibatches, eb.group_size):
        sub = [eps[i] for i in idx]
        groups = _groups_of(np.asarray(idx), eps, eb.group_size) if share_prompt else None
        if groups is not None:
            lead = [g[0] for g in groups]
            rows = np.concatenate([np.arange(starts[i], starts[i + 1]) for i in lead])
            vis = eb.vision.select(torch.from_numpy(rows).to(eb.vision.tokens.device)) \
                if eb.vision is not None else None
            acts = []
            for g in groups:
                ga = []
                for i in g:
                    a = np.asarray(eps[i].action_tokens, np.int64)
                    if max_sequence_length:
                        a = a[:max(0, int(max_sequence_length) - eps[i].prompt_length)]
                    ga.append(a)
                acts.append(ga)
            batch, counts = pack_groups(model.spec, [np.asarray(eps[i].prompt_tokens, np.int64) for i in lead], acts,
                                        [eps[i].grids for i in lead], vis, device=model.device)
        else:
            rows = np.concatenate([np.arange(starts[i], starts[i + 1]) for i in idx])
            vis = eb.vision.select(torch.from_numpy(rows).to(eb.vision.tokens.device)) \
                if eb.vision is not None else None
            seqs = [np.asarray(e.full_tokens, np.int64) for e in sub]
            if max_sequence_length:
                seqs = [s[:int(max_sequence_length)] for s in seqs]
            batch, counts = pack_sequences(model.spec, seqs, [e.prompt_length for e in sub], [e.grids for e in sub],
                                           vis, device=model.device)
        samp = np.concatenate([np.asarray(e.action_logprobs[:c], np.float32) for e, c in zip(sub, counts)])
        out.append(MiniBatch(batch=batch, seq_index=idx, counts=counts,
                             adv_tok=token_advantages(adv_seq[torch.from_numpy(idx)], counts, model.device),
                             sampler_lp=torch.from_numpy(samp).to(model.device)))
    return out


def collect(env, tokenizer, model, ts, cfg: TrainerConfig, batch_size: Optional[int] = None, rng: int = 0, *,
            eos_id: Optional[int] = None, generator=None, task_offset: int = 0, row_offset: int = 0,
            keep_groups: Optional[Tuple[int, int]] = None) -> CollectResult:
    """Roll out one iteration and build the minibatches (reference ``collect``, ``core/ppo.py:51-92``).

    ``keep_groups=(g0, g1)``: the rollout covers ``batch_size`` groups (e.g. a tensor-parallel rollout that
    every rank runs identically) but this process trains on groups [g0, g1) only.
    """
    G = int(batch_size) if batch_size else int(cfg.groups_per_batch)
    eb = collect_episodes(env, tokenizer, model, sampling_config(cfg, eos_id), groups_per_batch=G,
                          group_size=cfg.group_size, seed=rng, task_offset=task_offset, generator=generator,
                          min_pixels=cfg.vlm_min_pixels, max_pixels=cfg.vlm_max_pixels,
                          max_sequence_length=cfg.max_sequence_length, row_offset=row_offset)
    if keep_groups is not None:
        all_rewards = torch.tensor([e.reward for e in eb.episodes], dtype=torch.float32)
        if cfg.adv_norm == "batch":
            full_adv = group_advantages(all_rewards, cfg.group_size, "batch")
        eb = eb.subset(keep_groups[0], keep_groups[1], model.spec.vision.spatial_merge_size)
        rewards = torch.tensor([e.reward for e in eb.episodes], dtype=torch.float32)
        gs = max(1, cfg.group_size)
        if cfg.adv_norm == "batch":
            adv = full_adv[keep_groups[0] * gs:keep_groups[1] * gs].to(model.device)
        else:
            adv = group_advantages(rewards, cfg.group_size, cfg.adv_norm).to(model.device)
        mbs = build_minibatches(model, eb, adv, _minibatch_count(cfg, len(eb.episodes)), cfg.max_sequence_length,
                                share_prompt=cfg.share_prompt)
        return CollectResult(episodes=eb, rewards=rewards, advantages=adv, minibatches=mbs)
    rewards = torch.tensor([e.reward for e in eb.episodes], dtype=torch.float32)
    if cfg.adv_norm == "batch" and _distributed():
        import torch.distributed as dist

        st = torch.tensor([float(rewards.sum()), float((rewards ** 2).sum()), float(rewards.numel())],
                          dtype=torch.float64, device=model.device)
        dist.all_reduce(st)
        mean = st[0] / st[2]
        std = (st[1] / st[2] - mean ** 2).clamp_min(0).sqrt()
        a = rewards.to(model.device, torch.float64) - mean
        adv = (a / std if std > 1e-8 else a).float()
    else:
        adv = group_advantages(rewards, cfg.group_size, cfg.adv_norm).to(model.device)
    mbs = build_minibatches(model, eb, adv, _minibatch_count(cfg, len(eb.episodes)), cfg.max_sequence_length,
                            share_prompt=cfg.share_prompt)
    return CollectResult(episodes=eb, rewards=rewards, advantages=adv, minibatches=mbs)


@torch.no_grad()
def score(model, mb: MiniBatch) -> torch.Tensor:
    logp, _, _ = model.token_logprobs(mb.batch, save=False)
    return logp


_TOKEN_METRICS = ("loss", "loss_pg", "loss_ent", "loss_kl", "entropy", "approx_kl", "clip_fraction",
                  "token_logprob_mean", "ref_kl")


def _distributed() -> bool:
    import torch.distributed as dist

    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def update(ts, cr: CollectResult, cfg: TrainerConfig, *, ref_model=None, kl_ctrl: Optional[AdaptiveKL] = None,
           kl_coef: Optional[float] = None) -> Tuple[Any, Dict[str, float]]:
    """PPO/GRPO epochs over the collected minibatches; returns (train_state, host metrics).

    Under data parallelism every rank holds its share of each minibatch; the
    loss is normalised by the GLOBAL number of scored tokens of the minibatch,
    so the summed (reduce-scattered) gradients equal the single-process
    gradient, and the token-mean metrics are summed across ranks.
    """
    import torch.distributed as dist

    model = ts.model
    distributed = _distributed()
    mbs = cr.minibatches
    use_policy_old = cfg.old_logprob_source == "policy"
    reuse_first = use_policy_old and cfg.ppo_epochs == 1
    with phase("score"):
        for i, mb in enumerate(mbs):
            if not use_policy_old:
                mb.old_lp = mb.sampler_lp
            elif not (reuse_first and i == 0):
                mb.old_lp = score(model, mb)
            if ref_model is not None and cfg.kl_ref_coef > 0:
                mb.ref_lp = score(ref_model, mb)
    coef = float(cfg.kl_coef if kl_coef is None else kl_coef)
    sums: Dict[str, torch.Tensor] = {}
    n = 0
    for _ in range(int(cfg.ppo_epochs)):
        for mb in mbs:
            logp, ent, ctx = model.token_logprobs(mb.batch, save=True)
            if mb.old_lp is None:
                mb.old_lp = logp.detach().clone()
            denom = None
            if distributed:
                cnt = torch.tensor([float(logp.numel())], device=logp.device)
                dist.all_reduce(cnt)
                denom = max(float(cnt.item()), 1e-8)
            _, g_lp, g_ent, m = ppo_loss(logp, ent, mb.old_lp, mb.adv_tok, clip_epsilon=cfg.clip_epsilon,
                                         entropy_coef=cfg.entropy_coef, kl_coef=coef, ref_logp=mb.ref_lp,
                                         kl_ref_coef=cfg.kl_ref_coef, denom=denom)
            if distributed:
                packed = torch.stack([m[k].float().reshape(()) for k in _TOKEN_METRICS])
                dist.all_reduce(packed)
                for i, k in enumerate(_TOKEN_METRICS):
                    m[k] = packed[i]
            with torch.no_grad():
                model.backward(ctx, g_lp, g_ent)
            del ctx
            with phase("optimizer"):
                m.update(ts.apply_gradients())
            if kl_ctrl is not None:
                coef = kl_ctrl.update(float(m["approx_kl"]), coef)
            for k, v in m.items():
                sums[k] = sums.get(k, 0.0) + v.detach().float()
            n += 1
    host = {k: float(v) / max(1, n) for k, v in sums.items()}
    host["kl_coef"] = coef
    return ts, host


__all__ = ["TrainerConfig", "MiniBatch", "CollectResult", "sampling_config", "build_minibatches", "collect", "score",
           "update"]
