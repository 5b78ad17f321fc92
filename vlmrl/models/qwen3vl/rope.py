"""Multimodal RoPE: position ids, frequency-axis assignment and cos/sin tables.

* ``get_rope_index`` — 3-axis (t, h, w) position ids of one token sequence with
  images (reference ``models/qwen3vl/model.py:230-347``; HF
  ``Qwen3VLModel.get_rope_index``).  Text runs advance all three axes together;
  an image of merged grid (t, h, w) placed at ``start`` takes
  ``(start + frame, start + row, start + col)`` and the next text position is
  ``start + max(t, h, w)``.  Returns ``(pos [3, T], delta)`` with
  ``delta = max(pos) + 1 - T``: decode positions are ``cache_len + delta``.
  Computed on the host in O(T) NumPy (the reference runs a per-row Python loop).
* ``mrope_axis_map`` — which axis drives each rotary frequency.  Interleaved
  (HF Qwen3-VL ``apply_interleaved_mrope``): index i uses H when ``i % 3 == 1``
  and ``i < 3*sec_h``, W when ``i % 3 == 2`` and ``i < 3*sec_w``, else T.
  Chunked (reference compat, ``model.py:118-129``): the first ``sec_t`` indices
  use T, the next ``sec_h`` H, the rest W.
* ``mrope_cos_sin`` — fp32 cos/sin ``[T, D]`` (rotate-half layout, the
  ``D/2`` frequencies duplicated) for the PyTorch path.  The CUDA kernels
  compute the same angles in-kernel from ``pos`` and never store tables.
* ``vision_rotary_pos`` — (row, col) patch coordinates in merge-window order
  for the ViT 2-D rotary embedding (HF ``Qwen3VLVisionModel.rot_pos_emb``).
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch


def get_rope_index(
    token_ids: Sequence[int] | np.ndarray,
    image_grids: Sequence[Tuple[int, int, int]],
    *,
    spatial_merge_size: int,
    image_token_id: int,
    video_token_id: Optional[int] = None,
    t_scale: Optional[Sequence[float]] = None,
) -> Tuple[np.ndarray, int]:
    """``t_scale[g]`` multiplies grid g's frame index (Qwen2.5-VL video: seconds per grid x tokens per
    second, truncated to an integer; images use 0); without it frame f takes index f."""
    ids = np.asarray(token_ids, dtype=np.int64).reshape(-1)
    n = ids.shape[0]
    pos = np.empty((3, n), dtype=np.int64)
    vision_ids = {int(image_token_id)} | ({int(video_token_id)} if video_token_id is not None else set())
    is_vis = np.isin(ids, list(vision_ids))
    grids = list(image_grids)
    gi = 0
    cur = 0
    i = 0
    while i < n:
        if not is_vis[i]:
            j = i
            while j < n and not is_vis[j]:
                j += 1
            pos[:, i:j] = cur + np.arange(j - i)[None, :]
            cur += j - i
            i = j
            continue
        if gi >= len(grids):
            raise ValueError("more image-token runs than image grids")
        t, h, w = (int(x) for x in grids[gi])
        gi += 1
        lt, lh, lw = t, h // spatial_merge_size, w // spatial_merge_size
        cnt = lt * lh * lw
        if i + cnt > n or not is_vis[i:i + cnt].all():
            raise ValueError(f"image token run at {i} shorter than its grid ({cnt} tokens)")
        tt, hh, ww = np.meshgrid(np.arange(lt), np.arange(lh), np.arange(lw), indexing="ij")
        if t_scale is not None:
            tt = (tt.astype(np.float64) * float(t_scale[gi - 1])).astype(np.int64)
        pos[0, i:i + cnt] = cur + tt.reshape(-1)
        pos[1, i:i + cnt] = cur + hh.reshape(-1)
        pos[2, i:i + cnt] = cur + ww.reshape(-1)
        cur = int(pos[:, i:i + cnt].max()) + 1
        i += cnt
    delta = int(pos.max()) + 1 - n if n else 0
    return pos, delta


def batch_rope_index(
    sequences: Sequence[Sequence[int]],
    grids_per_seq: Sequence[Sequence[Tuple[int, int, int]]],
    *,
    spatial_merge_size: int,
    image_token_id: int,
) -> Tuple[np.ndarray, np.ndarray]:
    """Packed positions ``[3, sum(T_i)]`` and per-sequence deltas ``[B]``."""
    outs, deltas = [], []
    for ids, grids in zip(sequences, grids_per_seq):
        p, d = get_rope_index(ids, grids, spatial_merge_size=spatial_merge_size, image_token_id=image_token_id)
        outs.append(p)
        deltas.append(d)
    packed = np.concatenate(outs, axis=1) if outs else np.zeros((3, 0), np.int64)
    return packed, np.asarray(deltas, dtype=np.int64)


def mrope_axis_map(rope_section: Sequence[int], half_dim: int, interleaved: bool) -> np.ndarray:
    sec = [int(s) for s in rope_section]
    axis = np.zeros(half_dim, dtype=np.int32)
    if len(sec) == 1:
        return axis
    if interleaved:
        for i in range(half_dim):
            if i % 3 == 1 and i < 3 * sec[1]:
                axis[i] = 1
            elif i % 3 == 2 and i < 3 * sec[2]:
                axis[i] = 2
    else:
        axis[sec[0]:sec[0] + sec[1]] = 1
        axis[sec[0] + sec[1]:] = 2
    return axis


def inv_freq(head_dim: int, theta: float) -> np.ndarray:
    half = head_dim // 2
    return (1.0 / (float(theta) ** (np.arange(0, half, dtype=np.float64) * 2.0 / head_dim))).astype(np.float32)


def mrope_cos_sin(pos: torch.Tensor, head_dim: int, theta: float, rope_section: Sequence[int],
                  interleaved: bool, scaling_factor: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """pos [3, T] (or [T]) -> cos, sin fp32 [T, head_dim]."""
    if pos.dim() == 1:
        pos = pos[None].expand(3, -1)
    half = head_dim // 2
    axis = torch.from_numpy(mrope_axis_map(rope_section, half, interleaved)).long().to(pos.device)
    freq = torch.from_numpy(inv_freq(head_dim, theta)).to(pos.device)
    p = pos.to(torch.float32)
    if scaling_factor:
        p = p / float(scaling_factor)
    sel = p[axis]                      # [half, T]
    ang = sel.t() * freq[None, :]      # [T, half]
    ang = torch.cat([ang, ang], dim=-1)
    return torch.cos(ang), torch.sin(ang)


def vision_rotary_pos(grids: Sequence[Tuple[int, int, int]], spatial_merge_size: int) -> np.ndarray:
    """[N, 2] (row, col) of every patch, in the merge-window order of the patch rows."""
    m = spatial_merge_size
    out: List[np.ndarray] = []
    for t, h, w in grids:
        hb, wb = h // m, w // m
        r = (np.arange(hb)[:, None, None, None] * m + np.arange(m)[None, None, :, None])
        c = (np.arange(wb)[None, :, None, None] * m + np.arange(m)[None, None, None, :])
        r = np.broadcast_to(r, (hb, wb, m, m)).reshape(-1)
        c = np.broadcast_to(c, (hb, wb, m, m)).reshape(-1)
        rc = np.stack([r, c], axis=-1)
        out.append(np.tile(rc, (int(t), 1)))
    return np.concatenate(out, axis=0) if out else np.zeros((0, 2), np.int64)


def vision_cos_sin(rc: torch.Tensor, head_dim: int, theta: float = 10000.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """ViT 2-D rotary: rotary dim = head_dim/2 split between rows and cols -> cos/sin [N, head_dim]."""
    rdim = head_dim // 2
    freq = 1.0 / (theta ** (torch.arange(0, rdim, 2, dtype=torch.float32, device=rc.device) / rdim))
    ang = torch.cat([rc[:, 0:1].float() * freq[None], rc[:, 1:2].float() * freq[None]], dim=-1)  # [N, rdim]
    ang = torch.cat([ang, ang], dim=-1)
    return torch.cos(ang), torch.sin(ang)


def pos_embed_interp_index(grids: Sequence[Tuple[int, int, int]], num_grid_per_side: int, spatial_merge_size: int):
    """Bilinear-interpolation indices/weights of the learned ViT position table.

    For each image the ``h x w`` patch grid samples the ``G x G`` table at
    ``linspace(0, G-1, h) x linspace(0, G-1, w)``; rows are then permuted into
    merge-window order and repeated over frames (HF ``fast_pos_embed_interpolate``).
    Returns (idx [4, N] int64, weight [4, N] fp32).
    """
    G, m = num_grid_per_side, spatial_merge_size
    idx_all, w_all = [], []
    for t, h, w in grids:
        hs = torch.linspace(0, G - 1, h).numpy()
        ws = torch.linspace(0, G - 1, w).numpy()
        h0, w0 = hs.astype(np.int64), ws.astype(np.int64)
        h1, w1 = np.minimum(h0 + 1, G - 1), np.minimum(w0 + 1, G - 1)
        dh, dw = (hs - h0).astype(np.float32), (ws - w0).astype(np.float32)
        idx = np.stack([
            (h0[:, None] * G + w0[None, :]), (h0[:, None] * G + w1[None, :]),
            (h1[:, None] * G + w0[None, :]), (h1[:, None] * G + w1[None, :]),
        ]).reshape(4, -1)
        wt = np.stack([
            (1 - dh)[:, None] * (1 - dw)[None, :], (1 - dh)[:, None] * dw[None, :],
            dh[:, None] * (1 - dw)[None, :], dh[:, None] * dw[None, :],
        ]).reshape(4, -1).astype(np.float32)
        # permute (h, w) -> (hb, wb, hm, wm)
        perm = np.arange(h * w).reshape(h // m, m, w // m, m).transpose(0, 2, 1, 3).reshape(-1)
        idx, wt = idx[:, perm], wt[:, perm]
        idx_all.append(np.tile(idx, (1, int(t))))
        w_all.append(np.tile(wt, (1, int(t))))
    return np.concatenate(idx_all, axis=1), np.concatenate(w_all, axis=1)


__all__ = ["get_rope_index", "batch_rope_index", "mrope_axis_map", "inv_freq", "mrope_cos_sin",
           "vision_rotary_pos", "vision_cos_sin", "pos_embed_interp_index"]
