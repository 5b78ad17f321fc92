"""Typed containers for sampling, batching and rollouts (reference ``core/types.py:19-111``).

``SamplingConfig`` / ``VLMInputs`` / ``SampleResult`` keep the reference fields.
``Batch`` is the packed varlen ``PackedBatch`` of the executor (tokens, MRoPE
positions, ``cu_seqlens``, vision rows, loss rows, targets) instead of padded
``[B, T]`` arrays with cos/sin tables.  ``Rollout`` keeps the reference fields
and adds GRPO group ids, sampler log-probs and per-token advantages.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Union

import numpy as np
import torch

from vlmrl.models.qwen3vl.model import PackedBatch, VisionEmbeddings

Batch = PackedBatch


@dataclass
class SamplingConfig:
    temperature: float = 1.0
    top_p: Optional[float] = None
    top_k: Optional[int] = None
    eos_id: Optional[int] = None
    pad_id: int = 0
    max_new_tokens: int = 64
    # the reference's decode start (reference core/sampling.py:248-288): the prefill logits are dropped and the
    # first decode step re-feeds each prompt's last token at position len(prompt), so the cache holds it twice
    compat_refeed_last_token: bool = False


@dataclass
class VLMInputs:
    """prompt_tokens: list of per-prompt id arrays (or a [B, T] tensor + pad id);
    vision: embeddings of all images in prompt order; grid_thw: per-prompt list of (t, h, w)."""
    prompt_tokens: Union[torch.Tensor, Sequence[np.ndarray]]
    vision: Optional[VisionEmbeddings]
    grid_thw: Sequence[Sequence[Sequence[int]]]
    image_pad_id: int


@dataclass
class SampleResult:
    tokens: torch.Tensor                 # [B, new] int64 (EOS-filled after the stop)
    logprobs: Optional[torch.Tensor]     # [B, new] fp32 sampler log-probs (0 after the stop)
    texts: List[str] = field(default_factory=list)
    lengths: Optional[torch.Tensor] = None   # [B] generated tokens up to and including EOS


@dataclass
class Rollout:
    tokens: List[np.ndarray]             # full sequences (prompt + action)
    old_logprobs: torch.Tensor           # [M] per scored token (policy at sampling time)
    returns: torch.Tensor                # [N] rewards
    mask_targets: torch.Tensor           # [M] 1.0 per scored action token
    prompt_lens: np.ndarray              # [N]
    action_lens: np.ndarray              # [N]
    texts: List[str] = field(default_factory=list)
    group_ids: Optional[np.ndarray] = None
    sampler_logprobs: Optional[torch.Tensor] = None   # [M]
    ref_logprobs: Optional[torch.Tensor] = None       # [M]
    advantages: Optional[torch.Tensor] = None         # [N]
    token_counts: Optional[np.ndarray] = None         # scored tokens per sequence


__all__ = ["SamplingConfig", "VLMInputs", "SampleResult", "Batch", "Rollout"]
