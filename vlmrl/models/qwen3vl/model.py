"""Qwen3-VL text decoder: explicit forward / backward executor over flat parameter units.

The decoder (HF ``Qwen3VLTextModel``; reference ``models/qwen3vl/model.py:425-884``)
is pre-norm: ``h += o_proj(attn(qk_norm_rope(qkv(rms(h)))))`` then
``h += down(swiglu(gate_up(rms(h))))``; vision embeddings replace the
``<|image_pad|>`` rows of the token embeddings and, after decoder layers
``0..len(deepstack)-1``, the deepstack features are added at the same rows.

Instead of autograd, ``forward_train`` records what each layer needs and
``backward_train`` runs the hand-written backward of every op in reverse,
writing weight gradients straight into per-unit fp32 flat buffers supplied by
the parameter source.  That is what lets FSDP reduce-scatter a unit's gradient
the moment its backward finishes (see ``vlmrl.parallel.fsdp``).

Design choices (vs. the reference):

* packed varlen token layout (``cu_seqlens``) — no padding in any kernel;
* the vocab projection only runs on rows whose target is in the loss mask,
  through the fused ``vocab_logprob`` op (logp, entropy, lse) that never
  materialises fp32 logits;
* the KV cache is ``[L, B, Hkv, Tmax, D]`` bf16, written by ``kv_write`` /
  the decode step; decode positions are ``cache_len + rope_delta``.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from vlmrl import ops
from vlmrl.ops import decode_step
from vlmrl.models.qwen3vl.config import Qwen3VLSpec
from vlmrl.models.qwen3vl.params import UnitLayout, all_layouts, text_layouts, vision_layout


# --------------------------------------------------------------------------- containers
@dataclass
class VisionEmbeddings:
    """Merged vision tokens (packed over images) and deepstack features of the same rows."""
    tokens: torch.Tensor
    deepstack: Tuple[torch.Tensor, ...] = ()

    @classmethod
    def concatenate(cls, embeds: Sequence["VisionEmbeddings"]) -> "VisionEmbeddings":
        if not embeds:
            return cls(tokens=torch.zeros(0, 0))
        n = len(embeds[0].deepstack)
        if any(len(e.deepstack) != n for e in embeds):
            raise ValueError("All VisionEmbeddings must have the same number of DeepStack levels to concatenate.")
        return cls(tokens=torch.cat([e.tokens for e in embeds], 0),
                   deepstack=tuple(torch.cat([e.deepstack[i] for e in embeds], 0) for i in range(n)))

    def cast(self, dtype) -> "VisionEmbeddings":
        return VisionEmbeddings(self.tokens.to(dtype), tuple(d.to(dtype) for d in self.deepstack))

    def to(self, device) -> "VisionEmbeddings":
        return VisionEmbeddings(self.tokens.to(device), tuple(d.to(device) for d in self.deepstack))

    def select(self, rows: torch.Tensor) -> "VisionEmbeddings":
        return VisionEmbeddings(self.tokens[rows], tuple(d[rows] for d in self.deepstack))


@dataclass
class PackedBatch:
    """Device-side packed sequences for the decoder.

    ``tokens``/``targets`` [T] int64 (targets only where ``loss_rows`` points),
    ``pos`` [3, T] int32, ``cu_seqlens`` [B+1] int32, ``vis_rows`` [R] int64
    (rows of ``<|image_pad|>`` tokens, in order), ``loss_rows`` [M] int64 rows
    whose next-token log-prob is scored (a row may repeat: with shared prompts
    the prompt's last row scores every member's first action token).
    ``pre``/``xq`` [segments, 2] int32 (optional): the shared-prefix key range
    of each segment and, inversely, the query rows outside a segment that
    attend to all of its keys (see ``vlmrl.core.batching.pack_groups``).
    """
    tokens: torch.Tensor
    pos: torch.Tensor
    cu_seqlens: torch.Tensor
    max_seqlen: int
    vis_rows: torch.Tensor
    loss_rows: torch.Tensor
    targets: torch.Tensor
    vision: Optional[VisionEmbeddings] = None
    pre: Optional[torch.Tensor] = None
    xq: Optional[torch.Tensor] = None


class KVCache:
    """Preallocated per-sequence KV cache ``[L, B, Hkv, Tmax, D]`` plus lengths ``[B]``."""

    def __init__(self, num_layers: int, batch: int, num_kv_heads: int, max_len: int, head_dim: int,
                 dtype=torch.bfloat16, device="cpu"):
        shape = (num_layers, batch, num_kv_heads, max_len, head_dim)
        self.keys = torch.zeros(shape, dtype=dtype, device=device)
        self.values = torch.zeros(shape, dtype=dtype, device=device)
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=device)
        # rows whose first share_len[b] entries equal row lead[b]'s (a group's shared prompt); decode
        # attention reads those from the leader's row.  Identity / 0 = no sharing.
        self.lead = torch.arange(batch, dtype=torch.int32, device=device)
        self.share_len = torch.zeros(batch, dtype=torch.int32, device=device)
        self.max_len = max_len
        self.block_table = None   # contiguous rows (see PagedKVCache)

    @classmethod
    def init(cls, batch, num_layers, num_heads, head_dim, max_len, dtype=torch.bfloat16, device="cpu"):
        return cls(num_layers, batch, num_heads, max_len, head_dim, dtype, device)

    def rows(self, layer: int):
        """(keys, values) of one layer as contiguous [B, Hkv, Tmax, D]."""
        return self.keys[layer], self.values[layer]


class PagedKVCache:
    """KV cache in 64-token blocks: pools ``keys`` / ``values`` [L, NB, Hkv, 64, D] and a block table
    ``block_table`` int32 [B, max_len / 64] naming, per sequence, the pool block of each 64-token span.

    ``assign(prompt_lens, group_size)`` lays a GRPO batch out: the members of a group point at their
    leader's full prompt blocks, so a prompt's keys and values are stored (and streamed by decode
    attention) once per group; every row owns the blocks from its prompt's last, partial block on.
    After the prefill has written the leaders' rows, ``copy_prompt_tails`` gives each member its own copy
    of that partial block.  The decode kernels (``dec_qkv`` append, ``decode_attn``) and the prefill's
    ``kv_write`` address through the table; the block pool and the table keep their addresses, so a
    captured decode graph replays against whatever layout ``assign`` wrote last.

    No reference counterpart: the reference keeps one contiguous row per sequence
    (``models/qwen3vl/model.py:633-687``)."""

    block_size = 64

    def __init__(self, num_layers: int, batch: int, num_kv_heads: int, max_len: int, head_dim: int,
                 num_blocks: int, dtype=torch.bfloat16, device="cpu"):
        bs = self.block_size
        if max_len % bs:
            raise ValueError(f"paged KV cache: max_len {max_len} must be a multiple of {bs}")
        self.blocks_per_row = max_len // bs
        self.num_blocks = int(num_blocks)
        shape = (num_layers, self.num_blocks, num_kv_heads, bs, head_dim)
        self.keys = torch.zeros(shape, dtype=dtype, device=device)
        self.values = torch.zeros(shape, dtype=dtype, device=device)
        self.block_table = torch.zeros(batch, self.blocks_per_row, dtype=torch.int32, device=device)
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=device)
        # sharing is expressed by the block table; the row-sharing fields stay identity / 0
        self.lead = torch.arange(batch, dtype=torch.int32, device=device)
        self.share_len = torch.zeros(batch, dtype=torch.int32, device=device)
        self.max_len = max_len
        self._tails = None

    @staticmethod
    def blocks_needed(prompt_lens, group_size: int, max_len: int) -> int:
        """Pool blocks ``assign`` uses for these prompts (one per group member per block from the prompt's
        partial block on, plus the leader's full prompt blocks)."""
        mb = max_len // PagedKVCache.block_size
        gs = max(1, int(group_size))
        n = 0
        for p in prompt_lens:
            full = min(int(p) // PagedKVCache.block_size, mb)
            n += full + gs * (mb - full)
        return n

    def assign(self, prompt_lens, group_size: int = 1) -> int:
        """Write the block table for prompts ``prompt_lens`` (rows ordered (prompt, member)); returns the
        number of pool blocks used."""
        bs, mb = self.block_size, self.blocks_per_row
        gs = max(1, int(group_size))
        B = self.block_table.shape[0]
        if len(prompt_lens) * gs != B:
            raise ValueError(f"{len(prompt_lens)} prompts x group {gs} != {B} cache rows")
        need = self.blocks_needed(prompt_lens, gs, self.max_len)
        if need > self.num_blocks:
            raise ValueError(f"paged KV cache: {need} blocks needed, pool has {self.num_blocks}")
        table = np.zeros((B, mb), dtype=np.int32)
        nxt = 0
        src, dst = [], []
        for g, p in enumerate(prompt_lens):
            full = min(int(p) // bs, mb)
            shared = np.arange(nxt, nxt + full, dtype=np.int32)
            nxt += full
            for j in range(gs):
                b = g * gs + j
                table[b, :full] = shared
                table[b, full:] = np.arange(nxt, nxt + mb - full, dtype=np.int32)
                nxt += mb - full
            if gs > 1 and full < mb and int(p) % bs:
                lead_tail = table[g * gs, full]
                for j in range(1, gs):
                    src.append(lead_tail)
                    dst.append(table[g * gs + j, full])
        self.block_table.copy_(torch.from_numpy(table))
        dev = self.keys.device
        self._tails = ((torch.tensor(src, dtype=torch.int64, device=dev), torch.tensor(dst, dtype=torch.int64, device=dev))
                       if src else None)
        return nxt

    def copy_prompt_tails(self) -> None:
        """Members get their own copy of the leader's partial prompt block (written by the prefill)."""
        if self._tails is None:
            return
        src, dst = self._tails
        for pool in (self.keys, self.values):
            pool.index_copy_(1, dst, pool.index_select(1, src))

    def rows(self, layer: int):
        """(keys, values) of one layer as contiguous [B, Hkv, max_len, D] (a gathered copy)."""
        return ops.paged_rows(self.keys[layer], self.block_table), ops.paged_rows(self.values[layer], self.block_table)


# VLMRL_DECODE_L2_PREFETCH=1: decode kernels ask the L2 to fetch the next GEMM's weights.  Off by default:
# on the 4B model at batch 64 it measured slower (4.70 vs 4.44 ms per step); the decode GEMMs are bound by
# their fixed pipeline latency, and the prefetched lines compete with the KV-cache stream for L2.
_DECODE_L2_PREFETCH = os.environ.get("VLMRL_DECODE_L2_PREFETCH", "0") == "1"
# VLMRL_DECODE_FUSED=1: decode GEMMs run their consumer (q/k/v, residual + norm, SwiGLU) in the same launch
# after a grid-wide barrier.  Off by default: measured slower (5.04 vs 4.10 ms per 4B decode step at batch
# 64) than the separate consumer kernels, which overlap the GEMM's tail through programmatic launch.
_DECODE_FUSED_CONSUMERS = os.environ.get("VLMRL_DECODE_FUSED", "0") == "1"


# --------------------------------------------------------------------------- parameter sources
class LocalParams:
    """Full parameter units resident on one device (no sharding).

    ``get(name)`` returns the unit's flat compute-dtype buffer; ``grad(name)``
    the fp32 gradient accumulator (allocated on first use) and
    ``grad_done(name)`` is the hook where a sharded source reduces gradients.
    """

    def __init__(self, units: Dict[str, torch.Tensor], trainable: Optional[Sequence[str]] = None):
        self.units = units
        self.trainable = set(trainable) if trainable is not None else set(units)
        self.grads: Dict[str, torch.Tensor] = {}

    def get(self, name: str) -> torch.Tensor:
        return self.units[name]

    def release(self, name: str) -> None:
        pass

    def grad(self, name: str) -> Optional[torch.Tensor]:
        if name not in self.trainable:
            return None
        g = self.grads.get(name)
        if g is None:
            g = torch.zeros(self.units[name].numel(), dtype=torch.float32, device=self.units[name].device)
            self.grads[name] = g
        return g

    def grad_done(self, name: str) -> None:
        pass

    def zero_grads(self) -> None:
        for g in self.grads.values():
            g.zero_()


# --------------------------------------------------------------------------- decoder
@dataclass
class _LayerCtx:
    x: torch.Tensor
    xn: torch.Tensor
    r1: torch.Tensor
    qkv: torch.Tensor
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    rq: torch.Tensor
    rk: torch.Tensor
    o: torch.Tensor
    lse: torch.Tensor
    h1: torch.Tensor
    hn: torch.Tensor
    r2: torch.Tensor
    act: torch.Tensor
    pre: torch.Tensor


@dataclass
class TrainCtx:
    batch: PackedBatch
    layers: List[_LayerCtx] = field(default_factory=list)
    h_loss: Optional[torch.Tensor] = None
    hn_loss: Optional[torch.Tensor] = None
    r_final: Optional[torch.Tensor] = None
    lse: Optional[torch.Tensor] = None
    ent: Optional[torch.Tensor] = None


class TextDecoder:
    def __init__(self, spec: Qwen3VLSpec):
        self.spec = spec
        t = spec.text
        self.t = t
        self.H, self.D = t.hidden_size, t.head_dim
        self.nq, self.nkv = t.num_attention_heads, t.num_key_value_heads
        self.eps = t.rms_norm_eps
        self.scale = 1.0 / math.sqrt(t.head_dim)
        self.rope = ops.RopeCfg(t.head_dim, t.rope_theta, t.rope_section, t.mrope_interleaved)
        self.layouts = {l.name: l for l in text_layouts(spec)}
        self.n_layers = t.num_hidden_layers

    # ---------------------------------------------------------------- helpers
    def _w(self, params, name: str) -> Dict[str, torch.Tensor]:
        views = getattr(params, "views", None)     # sharded sources hand out gather-on-use weights
        if views is not None:
            v = views(name, self.layouts[name])
            if v is not None:
                return v
        return self.layouts[name].views(params.get(name))

    def _g(self, params, name: str) -> Optional[Dict[str, torch.Tensor]]:
        g = params.grad(name)
        return None if g is None else self.layouts[name].views(g)

    def embed_inputs(self, params, batch: PackedBatch) -> torch.Tensor:
        e = self._w(params, "embed")["embed"]
        h = ops.embed(batch.tokens, e)
        if batch.vision is not None and batch.vis_rows.numel():
            ops.scatter_rows_(h, batch.vis_rows, batch.vision.tokens.to(h.dtype), add=False)
        params.release("embed")
        return h

    def _deepstack(self, h, batch: PackedBatch, i: int):
        if batch.vision is not None and i < len(batch.vision.deepstack) and batch.vis_rows.numel():
            ops.scatter_rows_(h, batch.vis_rows, batch.vision.deepstack[i].to(h.dtype), add=True)
        return h

    # ---------------------------------------------------------------- layer fwd
    def layer_forward(self, w: Dict[str, torch.Tensor], x: torch.Tensor, pos: torch.Tensor, cu: torch.Tensor,
                      max_seqlen: int, save: bool, kv_sink=None, pre=None):
        T = x.shape[0]
        xn, r1 = ops.rms_norm(x, w["input_norm"], self.eps)
        qkv = ops.linear(xn, w["qkv_w"], bias=w["qkv_b"], out_dtype=x.dtype)
        q, k, v, rq, rk = ops.qk_norm_rope(qkv, w.get("q_norm"), w.get("k_norm"), pos, self.rope,
                                           n_q=self.nq, n_kv=self.nkv, eps=self.eps)
        if kv_sink is not None:
            kv_sink(k, v)
        o, lse = ops.flash_attn(q, k, v, cu, max_seqlen, causal=True, scale=self.scale, pre=pre)
        h1 = ops.linear(o.reshape(T, self.nq * self.D), w["o_w"], residual=x, out_dtype=x.dtype)
        hn, r2 = ops.rms_norm(h1, w["post_norm"], self.eps)
        act, pre = ops.linear_swiglu(hn, w["gu_w"], save_pre=save)
        out = ops.linear(act, w["down_w"], residual=h1, out_dtype=x.dtype)
        ctx = _LayerCtx(x, xn, r1, qkv, q, k, v, rq, rk, o, lse, h1, hn, r2, act, pre) if save else None
        return out, ctx

    # ---------------------------------------------------------------- layer bwd
    def layer_backward(self, w, g, c: _LayerCtx, dy: torch.Tensor, pos, cu, max_seqlen, pre=None,
                       xq=None) -> torch.Tensor:
        T = dy.shape[0]
        dt = dy.dtype
        # MLP
        if g is not None:
            ops.grad_weight(dy, c.act, accumulate=g["down_w"])
        d_pre = ops.grad_input_swiglu(dy, w["down_w"], c.pre)
        if g is not None:
            ops.grad_weight(d_pre, c.hn, accumulate=g["gu_w"])
        d_hn = ops.grad_input(d_pre, w["gu_w"], out_dtype=dt)
        d_h1 = ops.rms_norm_bwd(d_hn, c.h1, w["post_norm"], c.r2, dw_accum=None if g is None else g["post_norm"],
                                add=dy)
        # attention
        o2 = c.o.reshape(T, self.nq * self.D)
        if g is not None:
            ops.grad_weight(d_h1, o2, accumulate=g["o_w"])
        d_o = ops.grad_input(d_h1, w["o_w"], out_dtype=dt).view(T, self.nq, self.D)
        dq, dk, dv = ops.flash_attn_bwd(d_o, c.q, c.k, c.v, c.o, c.lse, cu, max_seqlen, causal=True, scale=self.scale,
                                        pre=pre, xq=xq)
        d_qkv = ops.qk_norm_rope_bwd(dq, dk, dv, c.qkv, w.get("q_norm"), w.get("k_norm"), pos, c.rq, c.rk, self.rope,
                                     n_q=self.nq, n_kv=self.nkv, eps=self.eps,
                                     dqw_accum=None if g is None else g.get("q_norm"),
                                     dkw_accum=None if g is None else g.get("k_norm"))
        if g is not None:
            ops.grad_weight(d_qkv, c.xn, accumulate=g["qkv_w"])
            g["qkv_b"].add_(d_qkv.sum(0, dtype=torch.float32))  # fp32 accumulation, no fp32 copy of d_qkv
        d_xn = ops.grad_input(d_qkv, w["qkv_w"], out_dtype=dt)
        return ops.rms_norm_bwd(d_xn, c.x, w["input_norm"], c.r1, dw_accum=None if g is None else g["input_norm"],
                                add=d_h1)

    # ---------------------------------------------------------------- full passes
    def hidden_states(self, params, batch: PackedBatch, *, save: bool = False, ctx: Optional[TrainCtx] = None,
                      kv_writer=None) -> torch.Tensor:
        h = self.embed_inputs(params, batch)
        for i in range(self.n_layers):
            w = self._w(params, f"layer{i}")
            sink = (lambda k, v, i=i: kv_writer(i, k, v)) if kv_writer is not None else None
            h, lc = self.layer_forward(w, h, batch.pos, batch.cu_seqlens, batch.max_seqlen, save, sink, batch.pre)
            params.release(f"layer{i}")
            if ctx is not None:
                ctx.layers.append(lc)
            h = self._deepstack(h, batch, i)
        return h

    def forward_logprobs(self, params, batch: PackedBatch, *, save: bool = False):
        """Per-loss-row (logp, entropy); with ``save`` also the TrainCtx for ``backward``."""
        ctx = TrainCtx(batch=batch) if save else None
        h = self.hidden_states(params, batch, save=save, ctx=ctx)
        head = self._w(params, "head")
        hs = h.index_select(0, batch.loss_rows)
        hn, r = ops.rms_norm(hs, head["final_norm"], self.eps)
        logp, ent, lse = ops.vocab_logprob(hn, head["lm_head"], batch.targets)
        params.release("head")
        if ctx is not None:
            ctx.h_loss, ctx.hn_loss, ctx.r_final, ctx.lse, ctx.ent = hs, hn, r, lse, ent
        return logp, ent, ctx

    def backward(self, params, ctx: TrainCtx, g_logp: torch.Tensor, g_ent: torch.Tensor) -> None:
        """Accumulate parameter gradients of ``sum(g_logp*logp + g_ent*entropy)``."""
        b = ctx.batch
        head = self._w(params, "head")
        gh = self._g(params, "head")
        dw_lm = gh["lm_head"] if gh is not None else torch.zeros_like(head["lm_head"], dtype=torch.float32)
        d_hn = ops.vocab_logprob_bwd(ctx.hn_loss, head["lm_head"], b.targets, ctx.lse, ctx.ent,
                                     g_logp.float().contiguous(), g_ent.float().contiguous(), dw_lm)
        d_hs = ops.rms_norm_bwd(d_hn, ctx.h_loss, head["final_norm"], ctx.r_final,
                                dw_accum=None if gh is None else gh["final_norm"])
        params.grad_done("head")
        params.release("head")
        T = b.tokens.shape[0]
        if b.pre is not None:   # loss rows may repeat (shared prompt rows): sum their gradients in fp32
            dh = torch.zeros(T, self.H, dtype=torch.float32, device=d_hs.device)
            dh.index_add_(0, b.loss_rows, d_hs.float())
            dh = dh.to(d_hs.dtype)
        else:
            dh = torch.zeros(T, self.H, dtype=d_hs.dtype, device=d_hs.device)
            dh.index_copy_(0, b.loss_rows, d_hs)
        for i in reversed(range(self.n_layers)):
            w = self._w(params, f"layer{i}")
            g = self._g(params, f"layer{i}")
            dh = self.layer_backward(w, g, ctx.layers[i], dh, b.pos, b.cu_seqlens, b.max_seqlen, b.pre, b.xq)
            ctx.layers[i] = None
            params.grad_done(f"layer{i}")
            params.release(f"layer{i}")
        ge = self._g(params, "embed")
        if ge is not None:
            toks = b.tokens
            if b.vision is not None and b.vis_rows.numel():
                toks = toks.clone()
                toks[b.vis_rows] = -1            # injected rows carry no embedding gradient
            ops.embed_bwd(toks, dh, ge["embed"])
            params.grad_done("embed")

    # ---------------------------------------------------------------- inference
    def final_logits(self, params, h_rows: torch.Tensor, normed: bool = False) -> torch.Tensor:
        head = self._w(params, "head")
        hn = h_rows if normed else ops.rms_norm(h_rows, head["final_norm"], self.eps)[0]
        logits = ops.lm_logits(hn, head["lm_head"])
        params.release("head")
        return logits

    def prefill(self, params, batch: PackedBatch, cache: KVCache, slots: torch.Tensor) -> torch.Tensor:
        """Run the prompt, fill the KV cache rows ``slots[b]`` and return last-token logits [B, V] fp32."""
        cu = batch.cu_seqlens
        lens = (cu[1:] - cu[:-1]).to(torch.int64)
        T = batch.tokens.shape[0]
        seq_of_tok = torch.repeat_interleave(torch.arange(lens.numel(), device=cu.device), lens)
        pos_in_seq = torch.arange(T, device=cu.device) - cu[:-1].to(torch.int64)[seq_of_tok]
        slot_of_tok = slots.to(torch.int64)[seq_of_tok]

        def writer(i, k, v):
            ops.kv_write(k, v, cache.keys[i], cache.values[i], slot_of_tok, pos_in_seq, cache.block_table)

        h = self.hidden_states(params, batch, save=False, kv_writer=writer)
        last = (cu[1:].to(torch.int64) - 1)
        cache.lengths[slots.long()] = lens.to(torch.int32)
        return self.final_logits(params, h.index_select(0, last))

    def decode_hidden(self, params, tokens: torch.Tensor, cache: KVCache, rope_delta: torch.Tensor):
        """One decode step for all B cache rows; appends k, v at ``cache.lengths`` (not advanced here).

        Returns ``(h, normed)``: on a GPU the step runs the fused path (stream-K GEMM partials consumed by
        kernels that also do bias / q-k norm / RoPE / KV write, residual + RMSNorm, SwiGLU) and ``h`` is
        already normalised by ``final_norm``; on the CPU ``h`` is the raw residual stream.
        """
        e = self._w(params, "embed")["embed"]
        B = tokens.shape[0]
        if tokens.is_cuda and cache.block_table is None and self._persistent_ok(params, B):
            plan = decode_step.plan_for(self, params, cache, B)
            ops.embed(tokens, e, out=plan.x)
            params.release("embed")
            plan.xn.copy_(ops.rms_norm(plan.x, self._w(params, "layer0")["input_norm"], self.eps)[0])
            return plan.run(cache.lengths, rope_delta.to(torch.int64), cache.lead, cache.share_len), True
        x = ops.embed(tokens, e)
        params.release("embed")
        if tokens.is_cuda:
            return self._decode_fused(params, x, cache, rope_delta), True
        p1 = (cache.lengths.to(torch.int64) + rope_delta.to(torch.int64)).to(torch.int32)
        pos = p1[None].expand(3, B).contiguous()
        rows = torch.arange(B, device=tokens.device)
        cur = cache.lengths.to(torch.int64)
        lens_after = cache.lengths + 1
        for i in range(self.n_layers):
            w = self._w(params, f"layer{i}")
            xn, _ = ops.rms_norm(x, w["input_norm"], self.eps)
            qkv = ops.linear(xn, w["qkv_w"], bias=w["qkv_b"], out_dtype=x.dtype)
            q, k, v, _, _ = ops.qk_norm_rope(qkv, w.get("q_norm"), w.get("k_norm"), pos, self.rope,
                                             n_q=self.nq, n_kv=self.nkv, eps=self.eps)
            ops.kv_write(k, v, cache.keys[i], cache.values[i], rows, cur, cache.block_table)
            o = ops.decode_attn(q, cache.keys[i], cache.values[i], lens_after, scale=self.scale,
                                block_table=cache.block_table)
            h1 = ops.linear(o.reshape(B, self.nq * self.D), w["o_w"], residual=x, out_dtype=x.dtype)
            hn, _ = ops.rms_norm(h1, w["post_norm"], self.eps)
            act, _ = ops.linear_swiglu(hn, w["gu_w"], save_pre=False)
            x = ops.linear(act, w["down_w"], residual=h1, out_dtype=x.dtype)
            params.release(f"layer{i}")
        return x, False

    def _persistent_ok(self, params, B: int) -> bool:
        """The persistent decode step applies: enabled, supported shape, resident bf16 weights, and none of
        the per-kernel path's experiment switches set."""
        if not decode_step.ENABLED or _DECODE_L2_PREFETCH or _DECODE_FUSED_CONSUMERS:
            return False
        if not decode_step.supported(self.spec.text, B):
            return False
        w = self._w(params, "layer0")["qkv_w"]
        return torch.is_tensor(w) and w.dtype == torch.bfloat16

    def _decode_fused(self, params, x: torch.Tensor, cache: KVCache, rope_delta: torch.Tensor) -> torch.Tensor:
        B = x.shape[0]
        lens = cache.lengths
        delta = rope_delta.to(torch.int64)
        lens_after = lens + 1
        w = self._w(params, "layer0")
        xn, _ = ops.rms_norm(x, w["input_norm"], self.eps)
        # Optional L2 prefetch plan (see _DECODE_L2_PREFETCH): o_proj during the q/k/v consumer, the first
        # half of gate/up during attention and the rest during the o_proj consumer, down during SwiGLU, the
        # next layer's qkv during the closing residual + norm.
        pf = _DECODE_L2_PREFETCH
        bt = cache.block_table
        fused = _DECODE_FUSED_CONSUMERS and not pf and bt is None   # the in-GEMM consumers address rows only
        for i in range(self.n_layers):
            w = self._w(params, f"layer{i}")
            nxt_w = self._w(params, f"layer{i + 1}") if i + 1 < self.n_layers else None
            nxt = nxt_w["input_norm"] if nxt_w is not None else self._w(params, "head")["final_norm"]
            if fused:
                # four launches + attention per layer: each consumer runs inside its GEMM
                q = ops.dec_linear_qkv(xn, w["qkv_w"], w["qkv_b"], w.get("q_norm"), w.get("k_norm"), lens, delta,
                                       self.rope, cache.keys[i], cache.values[i], n_q=self.nq, n_kv=self.nkv,
                                       eps=self.eps)
                o = ops.decode_attn(q, cache.keys[i], cache.values[i], lens_after, scale=self.scale,
                                    lead=cache.lead, share_len=cache.share_len)
                h1, hn = ops.dec_linear_residual_norm(o.reshape(B, self.nq * self.D), w["o_w"], x, w["post_norm"],
                                                      self.eps)
                act = ops.dec_linear_swiglu(hn, w["gu_w"])
                x, xn = ops.dec_linear_residual_norm(act, w["down_w"], h1, nxt, self.eps)
                params.release(f"layer{i}")
                continue
            gu = w["gu_w"].reshape(-1)
            half = (gu.numel() // 2) // 128 * 128
            ws, meta = ops.gemm_partials(xn, w["qkv_w"])
            q = ops.dec_qkv(ws, meta, w["qkv_b"], w.get("q_norm"), w.get("k_norm"), lens, delta, self.rope,
                            cache.keys[i], cache.values[i], n_q=self.nq, n_kv=self.nkv, eps=self.eps,
                            prefetch=w["o_w"] if pf else None, block_table=bt)
            o = ops.decode_attn(q, cache.keys[i], cache.values[i], lens_after, scale=self.scale,
                                prefetch=gu[:half] if pf else None, lead=cache.lead, share_len=cache.share_len,
                                block_table=bt)
            ws, meta = ops.gemm_partials(o.reshape(B, self.nq * self.D), w["o_w"])
            h1, hn = ops.dec_residual_norm(ws, meta, x, w["post_norm"], self.eps, prefetch=gu[half:] if pf else None)
            ws, meta = ops.gemm_partials(hn, w["gu_w"])
            act = ops.dec_swiglu(ws, meta, prefetch=w["down_w"] if pf else None)
            ws, meta = ops.gemm_partials(act, w["down_w"])
            x, xn = ops.dec_residual_norm(ws, meta, h1, nxt, self.eps,
                                          prefetch=nxt_w["qkv_w"] if pf and nxt_w is not None else None)
            params.release(f"layer{i}")
        return xn


__all__ = ["VisionEmbeddings", "PackedBatch", "KVCache", "PagedKVCache", "LocalParams", "TextDecoder", "TrainCtx"]
