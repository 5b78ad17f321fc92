"""Padding helpers (reference API) and the packed varlen batch builders used by the kernels.

Reference-compatible helpers (``core/batching.py:49-193``): ``pad_sequences``,
``pad_float_sequences``, ``pad_vision``, ``pad_grid``, ``build_masks`` (target
mask over ``tokens[:, 1:]`` selecting ``action_len`` positions starting at
``prompt_len - 1``).  ``VLMRL_SKIP_DEEPSTACK=1`` drops deepstack levels as in
the reference.

Packed builders (new): ``pack_rows`` turns ``[B, T]`` tokens + mask into a
``PackedBatch``; ``pack_sequences`` turns per-episode token arrays (prompt +
action) into the training batch: inputs ``s[:-1]``, targets ``s[1:]`` and loss
rows exactly where ``build_masks`` would put ones.  Position ids come from the
host-side ``get_rope_index`` and travel to the device with the tokens in one
pinned copy.
"""

from __future__ import annotations

import os
from typing import List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from vlmrl.models.qwen3vl.config import Qwen3VLSpec
from vlmrl.models.qwen3vl.model import PackedBatch, VisionEmbeddings
from vlmrl.models.qwen3vl.rope import get_rope_index

_SKIP_DEEPSTACK = os.environ.get("VLMRL_SKIP_DEEPSTACK", "0") == "1"


def set_skip_deepstack(flag: bool) -> None:
    global _SKIP_DEEPSTACK
    _SKIP_DEEPSTACK = bool(flag)


def pad_sequences(seqs: Sequence[np.ndarray], pad_val: int, max_len: Optional[int] = None) -> torch.Tensor:
    if not seqs:
        return torch.zeros(0, 0, dtype=torch.int32)
    T = max(len(s) for s in seqs)
    T = min(T, max_len) if max_len else T
    out = np.full((len(seqs), T), pad_val, dtype=np.int32)
    for i, s in enumerate(seqs):
        s = np.asarray(s, dtype=np.int32)[:T]
        out[i, :len(s)] = s
    return torch.from_numpy(out)


def pad_float_sequences(seqs: Sequence[np.ndarray], pad_val: float = 0.0, max_len: Optional[int] = None) -> torch.Tensor:
    if not seqs:
        return torch.zeros(0, 0, dtype=torch.float32)
    T = max(len(s) for s in seqs)
    T = min(T, max_len) if max_len else T
    out = np.full((len(seqs), T), pad_val, dtype=np.float32)
    for i, s in enumerate(seqs):
        s = np.asarray(s, dtype=np.float32)[:T]
        out[i, :len(s)] = s
    return torch.from_numpy(out)


def pad_vision(arrs: Sequence[Union[torch.Tensor, VisionEmbeddings]]):
    """[tokens_i, dim] list -> [B, max_tokens, dim] (zeros beyond each image's tokens)."""
    if not arrs:
        return torch.zeros(0, 0, 0)
    if isinstance(arrs[0], VisionEmbeddings):
        n = max(a.tokens.shape[0] for a in arrs)
        levels = 0 if _SKIP_DEEPSTACK else len(arrs[0].deepstack)

        def stack(get):
            first = get(arrs[0])
            out = torch.zeros(len(arrs), n, first.shape[-1], dtype=first.dtype, device=first.device)
            for i, a in enumerate(arrs):
                x = get(a)
                out[i, :x.shape[0]] = x
            return out

        for a in arrs:
            if levels and len(a.deepstack) != levels:
                raise ValueError("Inconsistent DeepStack depth across vision embeddings")
        return VisionEmbeddings(stack(lambda a: a.tokens), tuple(stack(lambda a, j=j: a.deepstack[j]) for j in range(levels)))
    n = max(a.shape[0] for a in arrs)
    out = torch.zeros(len(arrs), n, arrs[0].shape[-1], dtype=arrs[0].dtype)
    for i, a in enumerate(arrs):
        out[i, :a.shape[0]] = torch.as_tensor(a)
    return out


def pad_grid(arrs: Sequence[np.ndarray]) -> torch.Tensor:
    if not arrs:
        return torch.zeros(0, 0, 3, dtype=torch.int32)
    n = max(len(a) for a in arrs)
    out = np.zeros((len(arrs), n, 3), dtype=np.int32)
    for i, a in enumerate(arrs):
        a = np.asarray(a, dtype=np.int32).reshape(-1, 3)
        out[i, :len(a)] = a
    return torch.from_numpy(out)


def build_masks(prompt_lens: Sequence[int], action_lens: Sequence[int], seq_len: int) -> torch.Tensor:
    if seq_len <= 1:
        return torch.zeros(len(prompt_lens), 0, dtype=torch.int32)
    mask = np.zeros((len(prompt_lens), seq_len - 1), dtype=np.int32)
    for i, (p, a) in enumerate(zip(prompt_lens, action_lens)):
        p, a = int(p), int(a)
        if a <= 0:
            continue
        start = max(p - 1, 0)
        end = min(start + a - 1, seq_len - 2)
        if start <= end:
            mask[i, start:end + 1] = 1
    return torch.from_numpy(mask)


# --------------------------------------------------------------------------- packed builders
def _to_device(arrays: Sequence[np.ndarray], device) -> List[torch.Tensor]:
    """One pinned staging buffer, one H2D copy, then views (keeps small host->device traffic to one transfer)."""
    device = torch.device(device)
    flat = [np.ascontiguousarray(a, dtype=np.int64).reshape(-1) for a in arrays]
    sizes = [f.size for f in flat]
    host = torch.from_numpy(np.concatenate(flat) if flat else np.zeros(0, np.int64))
    if device.type == "cuda":
        host = host.pin_memory()
        dev = host.to(device, non_blocking=True)
    else:
        dev = host
    out, off = [], 0
    for a, n in zip(arrays, sizes):
        out.append(dev[off:off + n].view(np.asarray(a).shape))
        off += n
    return out


def pack_sequences(spec: Qwen3VLSpec, sequences: Sequence[np.ndarray], prompt_lens: Sequence[int],
                   grids_per_seq: Sequence[Sequence[Tuple[int, int, int]]], vision: Optional[VisionEmbeddings],
                   *, device="cpu", score_all: bool = False) -> Tuple[PackedBatch, np.ndarray]:
    """Training batch from full episodes (prompt + action tokens).

    Inputs are ``s[:-1]``, targets ``s[1:]``; loss rows are the action targets
    (rows ``prompt_len-1 .. len(s)-2``), or every row when ``score_all``.
    ``vision`` holds the image tokens of all sequences concatenated in order.
    Returns the batch and the per-sequence number of loss rows.
    """
    toks, poss, targ, vis, loss, counts, cu = [], [], [], [], [], [], [0]
    merge = spec.vision.spatial_merge_size if spec.vision is not None else 1
    for s, p, grids in zip(sequences, prompt_lens, grids_per_seq):
        s = np.asarray(s, dtype=np.int64)
        inp = s[:-1]
        pos, _ = get_rope_index(inp, grids, spatial_merge_size=merge, image_token_id=spec.image_token_id)
        base = cu[-1]
        toks.append(inp)
        poss.append(pos)
        vis.append(base + np.nonzero(inp == spec.image_token_id)[0])
        start = 0 if score_all else max(int(p) - 1, 0)
        rows = np.arange(start, len(inp))
        loss.append(base + rows)
        targ.append(s[1:][rows])
        counts.append(len(rows))
        cu.append(base + len(inp))
    tokens = np.concatenate(toks)
    pos = np.concatenate(poss, axis=1).astype(np.int64)
    t_tok, t_pos, t_cu, t_vis, t_loss, t_tgt = _to_device(
        [tokens, pos, np.asarray(cu, np.int64), np.concatenate(vis), np.concatenate(loss), np.concatenate(targ)], device)
    max_len = int(max(np.diff(cu))) if len(cu) > 1 else 0
    batch = PackedBatch(tokens=t_tok, pos=t_pos.to(torch.int32), cu_seqlens=t_cu.to(torch.int32), max_seqlen=max_len,
                        vis_rows=t_vis, loss_rows=t_loss, targets=t_tgt, vision=vision)
    return batch, np.asarray(counts)


def pack_groups(spec: Qwen3VLSpec, prompts: Sequence[np.ndarray], actions: Sequence[Sequence[np.ndarray]],
                grids_per_prompt: Sequence[Sequence[Tuple[int, int, int]]], vision: Optional[VisionEmbeddings],
                *, device="cpu") -> Tuple[PackedBatch, np.ndarray]:
    """Training batch where each prompt is computed once for all of its group's continuations.

    Group g packs as one prompt segment followed by one segment per member
    holding ``a_j[:-1]`` (the member's action tokens except the last).  Every
    member segment attends to its group's prompt keys (``pre``) and causally to
    itself; ``xq`` gives each prompt segment the query rows of its members (for
    the backward).  Member j's first action token is scored from the prompt's
    last row, the rest from its own rows, so the loss rows (and the per-member
    counts) come out in the same (group, member) order as ``pack_sequences``
    over the full sequences ``prompt + a_j``, with the same values: it is the
    same causal computation with the shared prefix done once.  ``vision`` holds
    the image tokens of each PROMPT once, in prompt order.
    """
    merge = spec.vision.spatial_merge_size if spec.vision is not None else 1
    toks, poss, vis, loss, targ, counts = [], [], [], [], [], []
    cu, pre, xq = [0], [], []
    for p, acts, grids in zip(prompts, actions, grids_per_prompt):
        p = np.asarray(p, dtype=np.int64)
        P = len(p)
        pos_p, delta = get_rope_index(p, grids, spatial_merge_size=merge, image_token_id=spec.image_token_id)
        p0 = cu[-1]
        toks.append(p)
        poss.append(pos_p)
        vis.append(p0 + np.nonzero(p == spec.image_token_id)[0])
        cu.append(p0 + P)
        pre.append((0, 0))
        seg_of_prompt = len(pre) - 1
        first_member = cu[-1]
        for a in acts:
            a = np.asarray(a, dtype=np.int64)
            R = len(a)
            counts.append(R)
            if R == 0:
                continue
            # first action token: scored from the prompt's last row
            rows = [p0 + P - 1]
            tg = [a[0]]
            if R > 1:
                base = cu[-1]
                inp = a[:-1]
                toks.append(inp)
                idx = P + np.arange(R - 1)
                poss.append(np.broadcast_to(idx + delta, (3, R - 1)).astype(np.int64))
                cu.append(base + R - 1)
                pre.append((p0, P))
                xq.append((0, 0))
                rows += list(base + np.arange(R - 1))
                tg += list(a[1:])
            loss.append(np.asarray(rows, np.int64))
            targ.append(np.asarray(tg, np.int64))
        xq.insert(seg_of_prompt, (first_member, cu[-1]))
    tokens = np.concatenate(toks)
    pos = np.concatenate(poss, axis=1).astype(np.int64)
    empty = np.zeros(0, np.int64)
    t_tok, t_pos, t_cu, t_vis, t_loss, t_tgt, t_pre, t_xq = _to_device(
        [tokens, pos, np.asarray(cu, np.int64), np.concatenate(vis) if vis else empty,
         np.concatenate(loss) if loss else empty, np.concatenate(targ) if targ else empty,
         np.asarray(pre, np.int64).reshape(-1, 2), np.asarray(xq, np.int64).reshape(-1, 2)], device)
    max_len = int(max(np.diff(cu))) if len(cu) > 1 else 0
    batch = PackedBatch(tokens=t_tok, pos=t_pos.to(torch.int32), cu_seqlens=t_cu.to(torch.int32), max_seqlen=max_len,
                        vis_rows=t_vis, loss_rows=t_loss, targets=t_tgt, vision=vision,
                        pre=t_pre.to(torch.int32), xq=t_xq.to(torch.int32))
    return batch, np.asarray(counts)


def pack_prompts(spec: Qwen3VLSpec, prompts: Sequence[np.ndarray], grids_per_seq, vision: Optional[VisionEmbeddings],
                 *, device="cpu") -> Tuple[PackedBatch, np.ndarray]:
    """Prefill batch: full prompts, no targets.  Returns (batch, rope deltas [B])."""
    toks, poss, vis, cu, deltas = [], [], [], [0], []
    merge = spec.vision.spatial_merge_size if spec.vision is not None else 1
    for s, grids in zip(prompts, grids_per_seq):
        s = np.asarray(s, dtype=np.int64)
        pos, d = get_rope_index(s, grids, spatial_merge_size=merge, image_token_id=spec.image_token_id)
        base = cu[-1]
        toks.append(s)
        poss.append(pos)
        vis.append(base + np.nonzero(s == spec.image_token_id)[0])
        deltas.append(d)
        cu.append(base + len(s))
    t_tok, t_pos, t_cu, t_vis = _to_device(
        [np.concatenate(toks), np.concatenate(poss, axis=1), np.asarray(cu, np.int64), np.concatenate(vis)], device)
    empty = t_vis[:0]
    batch = PackedBatch(tokens=t_tok, pos=t_pos.to(torch.int32), cu_seqlens=t_cu.to(torch.int32),
                        max_seqlen=int(max(np.diff(cu))), vis_rows=t_vis, loss_rows=empty, targets=empty, vision=vision)
    return batch, np.asarray(deltas, dtype=np.int64)


def pack_rows(spec: Qwen3VLSpec, tokens: torch.Tensor, attention_mask: Optional[torch.Tensor], grids_per_row,
              vision: Optional[VisionEmbeddings], device="cpu") -> Tuple[PackedBatch, torch.Tensor]:
    """``[B, T]`` tokens (+ mask) -> (PackedBatch over valid tokens, flat indices of those tokens in B*T)."""
    tok = tokens.detach().cpu().numpy()
    mask = np.ones_like(tok, dtype=bool) if attention_mask is None else attention_mask.detach().cpu().numpy().astype(bool)
    B = tok.shape[0]
    if grids_per_row is None:
        grids_rows = [[] for _ in range(B)]
    else:
        g = grids_per_row.tolist() if torch.is_tensor(grids_per_row) else grids_per_row
        if len(g) and not isinstance(g[0][0], (list, tuple)):
            # a flat list of grids in image order: distribute by each row's image count
            it = iter(g)
            grids_rows = []
            merge = spec.vision.spatial_merge_size
            for r in range(B):
                n_tok = int((tok[r][mask[r]] == spec.image_token_id).sum())
                rg = []
                while n_tok > 0:
                    t, h, w = next(it)
                    rg.append((t, h, w))
                    n_tok -= t * (h // merge) * (w // merge)
                grids_rows.append(rg)
        else:
            grids_rows = [[tuple(x) for x in row if any(x)] for row in g]
    seqs = [tok[r][mask[r]] for r in range(B)]
    batch, _ = pack_prompts(spec, seqs, grids_rows, vision, device=device)
    valid = torch.from_numpy(np.nonzero(mask.reshape(-1))[0]).to(device)
    return batch, valid


__all__ = ["pack_groups", "set_skip_deepstack", "pad_sequences", "pad_float_sequences", "pad_vision", "pad_grid", "build_masks",
           "pack_sequences", "pack_prompts", "pack_rows"]
