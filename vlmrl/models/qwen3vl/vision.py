"""Qwen3-VL vision tower executor (forward only; the tower is frozen during RL).

HF-faithful architecture (``transformers`` ``Qwen3VLVisionModel``), which the
reference approximates (reference ``models/qwen3vl/vision.py:178-331``; its
RMSNorm/SwiGLU/windowed variant is ``vision_arch="reference"``, below):

1. patch embedding: rows ``[N, C*Tp*P*P]`` -> ``[N, Hv]`` (Conv3d as one GEMM, with bias);
2. + bilinearly interpolated learned position embedding (merge-window order);
3. ``depth`` blocks: LayerNorm -> fused qkv (bias) -> 2-D rotary -> full
   bidirectional attention within each image -> proj (+residual) ->
   LayerNorm -> fc1 + GELU(tanh) -> fc2 (+residual);
4. after blocks in ``deepstack_visual_indexes``: a post-shuffle merger
   (2x2 concat -> LayerNorm(4Hv) -> fc1 -> GELU -> fc2) produces a deepstack feature;
5. final merger: LayerNorm(Hv) -> 2x2 concat -> fc1 -> GELU -> fc2 -> ``[N/4, out]``.

Every GEMM is ``vlmrl.ops.gemm`` (bias / GELU / residual fused in the epilogue)
and attention is ``vlmrl.ops.flash_attn`` over per-image ``cu_seqlens``.

``vision_arch == "qwen25"`` (HF Qwen2.5-VL, reference ``models/qwen25vl/vision.py``):
patch embedding without bias and without a position table; the patches are
permuted into attention windows of ``window_size`` pixels (merge units stay
together); blocks are RMSNorm -> qkv -> 2-D rotary -> attention within each
window (whole frame at ``fullatt_block_indexes``) -> proj, then RMSNorm ->
biased SwiGLU MLP; one merger (RMSNorm -> 2x2 concat -> fc1 -> GELU -> fc2);
the merged tokens are put back in raster order.

``vision_arch == "reference"`` (the Qwen3-VL tower as the reference computes it, reference
``models/qwen3vl/vision.py:178-331``): the qwen25 block structure with the reference's own
rotary pairing (``ops.vision_rope(style=1)``), windows of ``window_size`` pixels (one 2x2 merge unit
for Qwen3-VL configs, which give no window size), full attention over each whole image at
``fullatt_block_indexes`` (by default the deepstack indexes), a post-shuffle RMSNorm merger after
each deepstack block, and tanh-GELU in every merger; merged tokens and deepstack features are put
back in raster order.  The reference's full-attention ``cu_seqlens`` count ``4 * t*h*w`` tokens per
image (``vision.py:286-290``), which equals whole-image attention for the one image per call it
encodes; here each image is its own sequence for any batch of images.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from vlmrl import ops
from vlmrl.models.qwen3vl.config import Qwen3VLSpec
from vlmrl.models.qwen3vl.params import vision_layout
from vlmrl.models.qwen3vl.rope import pos_embed_interp_index, vision_rotary_pos


@dataclass
class VisionInputs:
    """Device-side metadata of a batch of images (built once per grid set)."""
    rc: torch.Tensor           # [N, 2] int32 (row, col) per patch
    pos_idx: torch.Tensor      # [4, N] int64 bilinear corners
    pos_w: torch.Tensor        # [4, N] fp32 weights
    cu_seqlens: torch.Tensor   # [images+1] int32
    max_seqlen: int
    # window attention (qwen25): patch order inside the tower, window cu_seqlens, merged-token inverse order
    perm: Optional[torch.Tensor] = None
    cu_window: Optional[torch.Tensor] = None
    max_window: int = 0
    unperm: Optional[torch.Tensor] = None


def window_index(grids: Sequence[Tuple[int, int, int]], merge: int, window_size: int, patch_size: int):
    """Merge units reordered window by window (row-major windows of ``window_size`` px per frame).

    Returns (order of merge units [U], cu_seqlens over patches of the windows).
    """
    ws = max(1, window_size // merge // patch_size)
    order, cu, off = [], [0], 0
    for t, h, w in grids:
        gh, gw = int(h) // merge, int(w) // merge
        index = np.arange(int(t) * gh * gw).reshape(int(t), gh, gw)
        for tt in range(int(t)):
            for r0 in range(0, gh, ws):
                for c0 in range(0, gw, ws):
                    blk = index[tt, r0:r0 + ws, c0:c0 + ws].reshape(-1)
                    order.append(blk + off)
                    cu.append(cu[-1] + blk.size * merge * merge)
        off += int(t) * gh * gw
    return (np.concatenate(order) if order else np.zeros(0, np.int64)), np.asarray(cu, np.int64)


def prepare_vision_inputs(spec: Qwen3VLSpec, grids: Sequence[Tuple[int, int, int]], device) -> VisionInputs:
    v = spec.vision
    rc = torch.from_numpy(vision_rotary_pos(grids, v.spatial_merge_size).astype(np.int32)).to(device)
    if v.num_position_embeddings:
        side = int(round(float(v.num_position_embeddings) ** 0.5))
        idx, w = pos_embed_interp_index(grids, side, v.spatial_merge_size)
        pos_idx, pos_w = torch.from_numpy(idx).to(device), torch.from_numpy(w).to(device)
    else:
        pos_idx = pos_w = torch.empty(0, device=device)
    lens = [int(t) * int(h) * int(w) for t, h, w in grids]
    # one attention sequence per frame (HF repeats h*w for each of the t frames)
    seq = []
    for t, h, w in grids:
        seq += [int(h) * int(w)] * int(t)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(seq)]).astype(np.int32), device=device)
    if spec.vision_arch == "reference":  # full-attention blocks span all frames of an image
        seq = [int(t) * int(h) * int(w) for t, h, w in grids]
        cu = torch.tensor(np.concatenate([[0], np.cumsum(seq)]).astype(np.int32), device=device)
    vin = VisionInputs(rc=rc, pos_idx=pos_idx, pos_w=pos_w, cu_seqlens=cu, max_seqlen=max(seq) if seq else 0)
    if spec.vision_arch in ("qwen25", "reference"):
        unit = v.spatial_merge_size ** 2
        order, cuw = window_index(grids, v.spatial_merge_size, v.window_size, v.patch_size)
        perm = (order[:, None] * unit + np.arange(unit)[None]).reshape(-1)
        vin.perm = torch.from_numpy(perm).to(device)
        vin.rc = vin.rc[vin.perm]
        vin.cu_window = torch.from_numpy(cuw.astype(np.int32)).to(device)
        vin.max_window = int(np.diff(cuw).max()) if len(cuw) > 1 else 0
        vin.unperm = torch.from_numpy(np.argsort(order)).to(device)
    return vin


class VisionTower:
    def __init__(self, spec: Qwen3VLSpec):
        if spec.vision is None:
            raise ValueError("spec has no vision tower")
        self.spec = spec
        self.v = spec.vision
        self.layout = vision_layout(spec)

    def _merge(self, x: torch.Tensor, p: Dict[str, torch.Tensor], prefix: str, post_norm: bool) -> torch.Tensor:
        M = self.v.merged_hidden_size
        eps = 1e-6
        if post_norm:
            x = ops.layer_norm(x.reshape(-1, M), p[prefix + "norm_w"], p[prefix + "norm_b"], eps)
        else:
            x = ops.layer_norm(x, p[prefix + "norm_w"], p[prefix + "norm_b"], eps).reshape(-1, M)
        h = ops.gemm(x, p[prefix + "fc1_w"], bias=p[prefix + "fc1_b"], epilogue=ops.EPI_GELU_ERF, out_dtype=x.dtype)
        return ops.gemm(h, p[prefix + "fc2_w"], bias=p[prefix + "fc2_b"], out_dtype=x.dtype)

    @torch.no_grad()
    def forward(self, flat: torch.Tensor, pixel_rows: torch.Tensor, vin: VisionInputs):
        """pixel_rows [N, patch_volume] -> (merged [N/4, out], [deepstack_k [N/4, out]])."""
        if self.spec.vision_arch == "qwen25":
            return self._forward_windowed(flat, pixel_rows, vin)[0], []
        if self.spec.vision_arch == "reference":
            return self._forward_windowed(flat, pixel_rows, vin)
        v = self.v
        p = self.layout.views(flat)
        dt = flat.dtype
        x = pixel_rows.to(dt)
        x = ops.gemm(x, p["patch_w"], bias=p["patch_b"], out_dtype=dt)
        if "pos_embed" in p and vin.pos_idx.numel():
            pe = (p["pos_embed"][vin.pos_idx].float() * vin.pos_w[..., None]).sum(0)
            x = (x.float() + pe).to(dt)
        H, nh = v.hidden_size, v.num_heads
        hd = H // nh
        deep_idx = list(v.deepstack_visual_indexes)
        deep: List[torch.Tensor] = []
        act = ops.EPI_GELU_TANH if "tanh" in v.hidden_act else ops.EPI_GELU_ERF
        for j in range(v.depth):
            b = f"b{j}."
            xn = ops.layer_norm(x, p[b + "n1_w"], p[b + "n1_b"], 1e-6)
            qkv = ops.gemm(xn, p[b + "qkv_w"], bias=p[b + "qkv_b"], out_dtype=dt)
            q, k, vv = ops.vision_rope(qkv, vin.rc, n_heads=nh, head_dim=hd)
            o, _ = ops.flash_attn(q, k, vv, vin.cu_seqlens, vin.max_seqlen, causal=False)
            x = ops.gemm(o.reshape(-1, H), p[b + "proj_w"], bias=p[b + "proj_b"], residual=x, out_dtype=dt)
            xn = ops.layer_norm(x, p[b + "n2_w"], p[b + "n2_b"], 1e-6)
            h = ops.gemm(xn, p[b + "fc1_w"], bias=p[b + "fc1_b"], epilogue=act, out_dtype=dt)
            x = ops.gemm(h, p[b + "fc2_w"], bias=p[b + "fc2_b"], residual=x, out_dtype=dt)
            if j in deep_idx:
                deep.append(self._merge(x, p, f"d{deep_idx.index(j)}.", post_norm=True))
        merged = self._merge(x, p, "m.", post_norm=False)
        return merged, deep

    def _forward_windowed(self, flat: torch.Tensor, pixel_rows: torch.Tensor, vin: VisionInputs):
        """RMSNorm/SwiGLU towers over window-ordered patches -> (merged, deepstack features), raster order."""
        v = self.v
        ref_tower = self.spec.vision_arch == "reference"
        p = self.layout.views(flat)
        dt = flat.dtype
        H, nh = v.hidden_size, v.num_heads
        hd = H // nh
        M = v.merged_hidden_size
        gelu = ops.EPI_GELU_TANH if ref_tower else ops.EPI_GELU_ERF
        x = ops.gemm(pixel_rows.to(dt), p["patch_w"], out_dtype=dt)
        x = x.index_select(0, vin.perm)
        full = set(int(i) for i in v.fullatt_block_indexes)
        deep_idx = list(v.deepstack_visual_indexes) if ref_tower else []
        deep: List[torch.Tensor] = []
        for j in range(v.depth):
            b = f"b{j}."
            cu, ms = (vin.cu_seqlens, vin.max_seqlen) if j in full else (vin.cu_window, vin.max_window)
            xn, _ = ops.rms_norm(x, p[b + "n1_w"], 1e-6)
            qkv = ops.gemm(xn, p[b + "qkv_w"], bias=p[b + "qkv_b"], out_dtype=dt)
            q, k, vv = ops.vision_rope(qkv, vin.rc, n_heads=nh, head_dim=hd, style=1 if ref_tower else 0)
            o, _ = ops.flash_attn(q, k, vv, cu, ms, causal=False)
            x = ops.gemm(o.reshape(-1, H), p[b + "proj_w"], bias=p[b + "proj_b"], residual=x, out_dtype=dt)
            xn, _ = ops.rms_norm(x, p[b + "n2_w"], 1e-6)
            a = ops.gemm(xn, p[b + "gu_w"], bias=p[b + "gu_b"], epilogue=ops.EPI_SWIGLU, out_dtype=dt)
            x = ops.gemm(a, p[b + "down_w"], bias=p[b + "down_b"], residual=x, out_dtype=dt)
            if j in deep_idx:  # post-shuffle merger: RMSNorm over the concatenated 2x2 unit
                pre = f"d{deep_idx.index(j)}."
                xn, _ = ops.rms_norm(x.reshape(-1, M), p[pre + "norm_w"], 1e-6)
                h = ops.gemm(xn, p[pre + "fc1_w"], bias=p[pre + "fc1_b"], epilogue=gelu, out_dtype=dt)
                deep.append(ops.gemm(h, p[pre + "fc2_w"], bias=p[pre + "fc2_b"], out_dtype=dt).index_select(0, vin.unperm))
        xn, _ = ops.rms_norm(x, p["m.norm_w"], 1e-6)
        h = ops.gemm(xn.reshape(-1, M), p["m.fc1_w"], bias=p["m.fc1_b"], epilogue=gelu, out_dtype=dt)
        merged = ops.gemm(h, p["m.fc2_w"], bias=p["m.fc2_b"], out_dtype=dt)
        return merged.index_select(0, vin.unperm), deep


__all__ = ["VisionInputs", "prepare_vision_inputs", "VisionTower"]
