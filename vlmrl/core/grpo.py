"""GRPO / PPO objective: group-relative advantages and the clipped loss with KL terms.

* ``group_advantages`` — GRPO: rewards are normalised within each group of
  ``group_size`` samples of the same prompt, ``(r - mean_g) / (std_g + eps)``.
  ``mode="batch"`` reproduces the reference's batch-wide normalisation
  (reference ``core/ppo.py:113-117``: centre over the batch, divide by the
  batch std only when it exceeds 1e-8; a single sample keeps its raw return).
* ``ppo_loss`` — per scored action token, with ``denom`` = number of scored
  tokens (reference ``core/ppo.py:133-177``):
  ``pg = max(-A*r, -A*clip(r, 1-eps, 1+eps))``, ``r = exp(logp - old)``;
  ``loss = mean(pg) - entropy_coef*mean(H) + kl_coef*mean(old - logp)``
  plus ``kl_ref_coef * mean(exp(ref - logp) - (ref - logp) - 1)`` — the k3
  estimator of KL(policy || frozen reference), the term the reference lacks.
  The gradient w.r.t. logp and entropy is taken with autograd on these small
  per-token vectors and handed to the model's explicit backward.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import numpy as np
import torch


def group_advantages(rewards: torch.Tensor, group_size: int, mode: str = "group", eps: float = 1e-6) -> torch.Tensor:
    r = rewards.float()
    if mode == "batch":
        if r.numel() <= 1:
            return r.clone()
        a = r - r.mean()
        std = a.std(unbiased=False)
        return a / std if std > 1e-8 else a
    if mode == "none":
        return r.clone()
    gs = max(1, int(group_size))
    if r.numel() % gs:
        raise ValueError(f"{r.numel()} rewards are not a multiple of group_size {gs}")
    g = r.view(-1, gs)
    a = g - g.mean(1, keepdim=True)
    return (a / (g.std(1, unbiased=False, keepdim=True) + eps)).reshape(-1)


def ppo_loss(logp: torch.Tensor, ent: torch.Tensor, old_logp: torch.Tensor, adv_tok: torch.Tensor, *,
             clip_epsilon: float, entropy_coef: float = 0.0, kl_coef: float = 0.0,
             ref_logp: Optional[torch.Tensor] = None, kl_ref_coef: float = 0.0,
             mask: Optional[torch.Tensor] = None, denom: Optional[float] = None):
    """Returns (loss, g_logp, g_ent, metrics) for the tokens of one minibatch."""
    lp = logp.detach().float().requires_grad_(True)
    en = ent.detach().float().requires_grad_(True)
    m = mask.float() if mask is not None else torch.ones_like(lp)
    d = float(denom) if denom is not None else m.sum().clamp_min(1e-8)
    old = old_logp.float()
    logratio = lp - old
    ratio = torch.exp(logratio)
    A = adv_tok.float()
    pg = torch.maximum(-A * ratio, -A * torch.clamp(ratio, 1 - clip_epsilon, 1 + clip_epsilon))
    loss_pg = (pg * m).sum() / d
    loss_ent = -float(entropy_coef) * (en * m).sum() / d
    kl_term = ((old - lp) * m).sum() / d
    loss_kl = float(kl_coef) * kl_term
    loss = loss_pg + loss_ent + loss_kl
    ref_kl = torch.zeros((), device=lp.device)
    if ref_logp is not None:
        x = ref_logp.float() - lp
        ref_kl = ((torch.exp(x) - x - 1.0) * m).sum() / d
        loss = loss + float(kl_ref_coef) * ref_kl
    loss.backward()
    with torch.no_grad():
        metrics = {
            "loss": loss.detach(), "loss_pg": loss_pg.detach(), "loss_ent": loss_ent.detach(),
            "loss_kl": loss_kl.detach() if torch.is_tensor(loss_kl) else torch.tensor(loss_kl),
            "entropy": (en.detach() * m).sum() / d,
            "approx_kl": (((ratio - 1.0) - logratio).detach() * m).sum() / d,
            "clip_fraction": (((ratio - 1.0).abs() > clip_epsilon).float().detach() * m).sum() / d,
            "token_logprob_mean": (lp.detach() * m).sum() / d,
            "ref_kl": ref_kl.detach(),
        }
    return loss.detach(), lp.grad, en.grad, metrics


def token_advantages(adv_seq: torch.Tensor, counts: np.ndarray, device) -> torch.Tensor:
    """Broadcast per-sequence advantages onto each sequence's scored tokens."""
    reps = torch.as_tensor(np.asarray(counts), dtype=torch.long, device=adv_seq.device)
    return torch.repeat_interleave(adv_seq, reps).to(device)


__all__ = ["group_advantages", "ppo_loss", "token_advantages"]
