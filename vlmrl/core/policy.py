"""Policy scoring and RoPE batch builder (reference ``core/policy.py:1-172``).

``token_logprobs_vlm`` scores every next token of right-padded ``[B, T]``
rows (``tokens[:, 1:]`` given ``tokens[:, :-1]``) and returns ``[B, T-1]``
fp32 log-probabilities, zero where ``token_mask`` is 0 — the reference's
contract.  Internally the rows are packed (no padding FLOPs) and scored by the
fused vocab log-prob kernel, which never materialises the logits.
``build_rope`` returns the interleaved-MRoPE cos/sin tables for a batch (the
kernels compute RoPE from position ids; the tables serve callers that want
them explicitly).  The reference's ``checkpoint`` flag (rematerialisation) is
accepted and ignored: the executor saves only per-layer inputs and recomputes
the rest in its backward.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple, Union

import numpy as np
import torch

from vlmrl.core.batching import pack_sequences
from vlmrl.models.qwen3vl.model import PackedBatch, VisionEmbeddings
from vlmrl.models.qwen3vl.rope import get_rope_index, mrope_cos_sin


def _model_of(obj):
    return getattr(obj, "model", obj)


def token_logprobs_vlm(train_state, image_pad_id: int, tokens: torch.Tensor, token_mask: torch.Tensor,
                       vision_embeds: Optional[VisionEmbeddings], grids: Sequence[Sequence[Tuple[int, int, int]]],
                       *, checkpoint: bool = False) -> torch.Tensor:
    """[B, T] tokens, [B, T-1] mask -> [B, T-1] log p(tokens[:, 1:]) (0 where masked)."""
    model = _model_of(train_state)
    spec = model.spec
    if int(image_pad_id) != int(spec.image_token_id):
        raise ValueError(f"image_pad_id {image_pad_id} does not match the model's {spec.image_token_id}")
    tok = torch.as_tensor(tokens).cpu().numpy()
    mask = torch.as_tensor(token_mask).cpu().numpy().astype(bool)
    B, T = tok.shape
    lens = [int(mask[b].sum()) + 1 if mask[b].any() else 1 for b in range(B)]
    seqs = [tok[b, :lens[b]] for b in range(B)]
    batch, counts = pack_sequences(spec, seqs, [1] * B, grids, vision_embeds, device=model.device, score_all=True)
    logp, _, _ = model.token_logprobs(batch, save=False)
    out = torch.zeros(B, T - 1, dtype=torch.float32, device=model.device)
    off = 0
    for b, c in enumerate(counts):
        out[b, :c] = logp[off:off + c]
        off += c
    return out * torch.as_tensor(token_mask, device=model.device).float()


def token_logprobs(train_state, image_pad_id: int, batch: PackedBatch, *, checkpoint: bool = False) -> torch.Tensor:
    """Log-probs of the loss rows of a packed batch (convenience wrapper, reference ``:80-97``)."""
    model = _model_of(train_state)
    logp, _, _ = model.token_logprobs(batch, save=False)
    return logp


def build_rope(spec, tokens: Union[np.ndarray, torch.Tensor], grids: Sequence[Sequence[Tuple[int, int, int]]],
               pad_id: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Right-padded [B, T] tokens -> (cos, sin) [B, T, head_dim] fp32 (reference ``build_rope``, ``:100-164``)."""
    tok = torch.as_tensor(tokens).cpu().numpy()
    B, T = tok.shape
    t = spec.text
    cos = torch.zeros(B, T, t.head_dim)
    sin = torch.zeros(B, T, t.head_dim)
    for b in range(B):
        valid = np.nonzero(tok[b] != pad_id)[0]
        n = int(valid[-1]) + 1 if len(valid) else 0
        if n == 0:
            continue
        pos, _ = get_rope_index(tok[b, :n], grids[b], spatial_merge_size=spec.vision.spatial_merge_size,
                                image_token_id=spec.image_token_id)
        c, s = mrope_cos_sin(torch.as_tensor(pos), t.head_dim, t.rope_theta, t.rope_section, t.mrope_interleaved)
        cos[b, :n], sin[b, :n] = c, s
    return cos, sin


__all__ = ["token_logprobs_vlm", "token_logprobs", "build_rope"]
