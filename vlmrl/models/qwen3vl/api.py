"""User-facing ``Qwen3VLModel``: parameters + vision tower + text decoder.

Method names follow the reference model (``models/qwen3vl/model.py:690-884``):
``encode_vision``, ``forward_text``, ``forward_vlm``, ``decode_step``; the RL
paths use ``token_logprobs`` (fused vocab op) and the executor's explicit
``backward``.  Inputs are batched ``[B, T]`` token tensors with an optional
attention mask; internally everything is packed (see ``vlmrl.core.batching``).
"""

from __future__ import annotations

import os

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from vlmrl import ops
from vlmrl.models.qwen3vl.config import Qwen3VLSpec
from vlmrl.models.qwen3vl.model import KVCache, LocalParams, PackedBatch, PagedKVCache, TextDecoder, VisionEmbeddings
from vlmrl.models.qwen3vl.params import all_layouts, init_params, text_layouts
from vlmrl.models.qwen3vl.vision import VisionTower, prepare_vision_inputs
from vlmrl.utils.vlm import CLIP_MEAN, CLIP_STD


# VLMRL_FUSED_SAMPLER=0: decode steps write the fp32 logits and sample them with the separate kernel.
_FUSED_SAMPLER = os.environ.get("VLMRL_FUSED_SAMPLER", "1") != "0"


class Qwen3VLModel:
    def __init__(self, spec: Qwen3VLSpec, *, units: Optional[Dict[str, torch.Tensor]] = None, params=None,
                 device="cpu", dtype=torch.bfloat16, seed: int = 0):
        self.spec = spec
        self.device = torch.device(device)
        self.dtype = dtype
        self.decoder = TextDecoder(spec)
        self.vision = VisionTower(spec) if spec.vision is not None else None
        if params is None:
            if units is None:
                units = init_params(spec, seed=seed, dtype=dtype, device=self.device)
            else:
                units = {k: v.detach().to(self.device, dtype, copy=True).contiguous() for k, v in units.items()}
            params = LocalParams(units, trainable=[l.name for l in text_layouts(spec)])
        self.params = params
        self._vin_cache: Dict[Tuple, object] = {}

    # ---------------------------------------------------------------- vision
    def vision_inputs(self, grids: Sequence[Tuple[int, int, int]]):
        key = tuple(tuple(int(x) for x in g) for g in grids)
        vin = self._vin_cache.get(key)
        if vin is None:
            vin = prepare_vision_inputs(self.spec, key, self.device)
            if len(self._vin_cache) > 16:
                self._vin_cache.clear()
            self._vin_cache[key] = vin
        return vin

    @torch.no_grad()
    def encode_vision(self, pixel_values: torch.Tensor, grid_thw) -> VisionEmbeddings:
        if self.vision is None:
            raise ValueError("Vision backbone not configured for this model")
        grids = [tuple(int(x) for x in g) for g in (grid_thw.tolist() if torch.is_tensor(grid_thw) else grid_thw)]
        flat = self.params.get("visual")
        merged, deep = self.vision.forward(flat, pixel_values.to(self.device), self.vision_inputs(grids))
        self.params.release("visual")
        return VisionEmbeddings(tokens=merged, deepstack=tuple(deep))

    @torch.no_grad()
    def encode_images_uint8(self, images: torch.Tensor) -> VisionEmbeddings:
        """Same-size uint8 images [N, H, W, 3] (H, W multiples of patch*merge) -> embeddings, patchified on device."""
        v = self.spec.vision
        N, H, W, _ = images.shape
        rows = ops.patchify_uint8(images.to(self.device), patch=v.patch_size, temporal=v.temporal_patch_size,
                                  merge=v.spatial_merge_size, mean=CLIP_MEAN.tolist(), std=CLIP_STD.tolist(),
                                  out_dtype=self.dtype)
        grids = [(1, H // v.patch_size, W // v.patch_size)] * N
        return self.encode_vision(rows, grids)

    # ---------------------------------------------------------------- text
    def _pack(self, tokens: torch.Tensor, attention_mask: Optional[torch.Tensor], grids_per_row,
              vision: Optional[VisionEmbeddings]):
        from vlmrl.core.batching import pack_rows

        return pack_rows(self.spec, tokens, attention_mask, grids_per_row, vision, device=self.device)

    @torch.no_grad()
    def forward_vlm(self, tokens: torch.Tensor, vision: Optional[VisionEmbeddings] = None, grid_thw=None,
                    attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Full fp32 logits ``[B, T, V]`` (zeros at masked positions).  Convenience/parity API."""
        batch, valid = self._pack(tokens, attention_mask, grid_thw, vision)
        h = self.decoder.hidden_states(self.params, batch)
        logits = self.decoder.final_logits(self.params, h)
        B, T = tokens.shape
        out = torch.zeros(B, T, logits.shape[-1], dtype=torch.float32, device=logits.device)
        out.view(B * T, -1)[valid] = logits.float()
        return out

    def forward_text(self, tokens: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.forward_vlm(tokens, None, None, attention_mask)

    __call__ = forward_text

    def token_logprobs(self, batch: PackedBatch, *, save: bool = False):
        return self.decoder.forward_logprobs(self.params, batch, save=save)

    def backward(self, ctx, g_logp, g_ent) -> None:
        self.decoder.backward(self.params, ctx, g_logp, g_ent)

    # ---------------------------------------------------------------- decoding
    def new_cache(self, batch: int, max_len: int, num_blocks: Optional[int] = None):
        """A contiguous ``KVCache``, or with ``num_blocks`` a ``PagedKVCache`` whose pool holds that many
        64-token blocks (lay it out with ``assign``)."""
        t = self.spec.text
        if num_blocks is not None:
            return PagedKVCache(t.num_hidden_layers, batch, t.num_key_value_heads, max_len, t.head_dim,
                                int(num_blocks), self.dtype, self.device)
        return KVCache(t.num_hidden_layers, batch, t.num_key_value_heads, max_len, t.head_dim, self.dtype, self.device)

    @torch.no_grad()
    def prefill(self, batch: PackedBatch, cache: KVCache, slots: torch.Tensor) -> torch.Tensor:
        return self.decoder.prefill(self.params, batch, cache, slots)

    @torch.no_grad()
    def decode_step(self, token: torch.Tensor, cache: KVCache, rope_deltas: torch.Tensor) -> torch.Tensor:
        """Logits [B, V] fp32 of the next token; appends this token's k/v and advances ``cache.lengths``."""
        h, normed = self.decoder.decode_hidden(self.params, token, cache, rope_deltas.reshape(-1))
        cache.lengths += 1
        return self.decoder.final_logits(self.params, h, normed=normed)

    def decode_step_sample(self, token: torch.Tensor, cache: KVCache, rope_deltas: torch.Tensor, *,
                           temperature: float, top_k: int, top_p: float, seed, step, row_offset: int = 0):
        """One decode step that returns the sampled (tokens, log-probs) directly; on a GPU with
        1 <= top_k <= 16 the lm_head and the top-k / top-p sampler are fused and no logits are written.
        Appends this token's k/v and advances ``cache.lengths``."""
        h, normed = self.decoder.decode_hidden(self.params, token, cache, rope_deltas.reshape(-1))
        cache.lengths += 1
        if h.is_cuda and _FUSED_SAMPLER and 1 <= int(top_k or 0) <= ops.FUSED_SAMPLER_MAX_TOPK:
            head = self.decoder._w(self.params, "head")
            hn = h if normed else ops.rms_norm(h, head["final_norm"], self.decoder.eps)[0]
            out = ops.lm_head_sample(hn, head["lm_head"], temperature=temperature, top_k=int(top_k), top_p=top_p,
                                     seed=seed, step=step, row_offset=row_offset)
            self.params.release("head")
            return out
        logits = self.decoder.final_logits(self.params, h, normed=normed)
        return ops.sample(logits, temperature=temperature, top_k=top_k or 0, top_p=top_p or 0.0, seed=seed, step=step,
                          row_offset=row_offset)

    def parameter_count(self, trainable_only: bool = False) -> int:
        return sum(l.numel for l in all_layouts(self.spec) if (l.trainable or not trainable_only))


__all__ = ["Qwen3VLModel"]
