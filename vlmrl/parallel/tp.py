"""Tensor-parallel decoding over the ranks of a process group (one GPU per rank, NVLink peers).

Every rank decodes the SAME batch of sequences with 1/W of each decoder layer's
weights (Megatron-style split, rebuilt for the decode step):

* q/k/v projections: column-parallel by attention head (rank r owns q heads
  ``[r*nq/W, (r+1)*nq/W)`` and kv heads ``[r*nkv/W, (r+1)*nkv/W)``); the KV
  cache holds only the local kv heads, so attention needs no communication;
* o_proj and down_proj: row-parallel; their stream-K partial sums are
  all-reduced INSIDE the residual + RMSNorm consumer kernel
  (``dec_residual_norm_tp``): each CTA stores its row of partials, every
  value tagged with the step epoch in one 8-byte word, into this rank's slot
  of every rank's IPC-shared buffer, polls its own buffer until all ranks'
  words carry the tag, and sums all ranks in rank order — so every rank ends
  with bitwise-identical activations, after one one-way NVLink store;
* gate/up: column-parallel (interleaved gate/up row pairs stay together);
* lm_head and sampler: vocab-parallel.  Rank r owns a contiguous shard of the
  vocabulary rows; its lm_head GEMM keeps each row's top-k per tile, its merge
  kernel finds the shard's top k, stores them (tagged with the step epoch) into
  every rank's slot and picks the global top k from all shards' survivors, so
  every rank draws the same token with the same Philox draw (``decode_step_sample``;
  ``decode_step`` still returns full logits from the replicated lm_head).
  Embedding and final norm are replicated.

The prefill runs replicated with the full weights (it is a small part of a
rollout); the local kv heads are then copied into the tensor-parallel cache.
Shards are re-sliced from the model's (gathered) parameters whenever they
changed (``refresh``), into buffers at fixed addresses so a captured decode
graph stays valid.  Synchronisation uses a device-side step counter (epoch)
advanced by the first kernel of every step; tags only grow, so nothing is
ever reset, and every wait is bounded (error code instead of a hang).

No reference counterpart: the reference decodes on one device
(``core/sampling.py:157-224``).
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from vlmrl import ops
from vlmrl.models.qwen3vl.model import KVCache
from vlmrl.ops._ext import ext

# VLMRL_FUSED_SAMPLER=0: sample from full logits (replicated lm_head) instead of the vocab-parallel path
_FUSED_SAMPLER = os.environ.get("VLMRL_FUSED_SAMPLER", "1") != "0"


class TPDecoder:
    def __init__(self, model, group=None, max_batch: int = 64):
        from vlmrl.parallel.symm import SymmetricBuffer

        self.model = model
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        spec = model.spec
        t = spec.text
        W = self.world
        for name, n in (("attention heads", t.num_attention_heads), ("kv heads", t.num_key_value_heads),
                        ("intermediate size", t.intermediate_size)):
            if n % W:
                raise ValueError(f"tensor parallelism over {W} ranks needs {name} ({n}) divisible by {W}")
        self.L, self.H, self.D = t.num_hidden_layers, t.hidden_size, t.head_dim
        self.nq, self.nkv, self.F = t.num_attention_heads, t.num_key_value_heads, t.intermediate_size
        self.nq_l, self.nkv_l, self.F_l = self.nq // W, self.nkv // W, self.F // W
        self.max_batch = int(max_batch)
        dev, dt = model.device, model.dtype
        L, H, D = self.L, self.H, self.D
        qkv_l = (self.nq_l + 2 * self.nkv_l) * D
        self.qkv_w = torch.empty(L, qkv_l, H, dtype=dt, device=dev)
        self.qkv_b = torch.empty(L, qkv_l, dtype=dt, device=dev)
        self.o_w = torch.empty(L, H, self.nq_l * D, dtype=dt, device=dev)
        self.gu_w = torch.empty(L, 2 * self.F_l, H, dtype=dt, device=dev)
        self.down_w = torch.empty(L, H, self.F_l, dtype=dt, device=dev)
        self.v0, self.v1 = vocab_shard(t.vocab_size, W, self.rank)
        self.lm_w = torch.empty(self.v1 - self.v0, H, dtype=dt, device=dev)
        # per rank: [W][max_batch][16 survivors][2] tagged words of the sampler exchange
        self.samp_slots = SymmetricBuffer(W * self.max_batch * ops.FUSED_SAMPLER_MAX_TOPK * 16, group, dev)
        self.points = 2 * L
        # per reduction point: [W source ranks][max_batch][H] tagged 8-byte words (zeroed: tags start at 1)
        self.point_bytes = W * self.max_batch * H * 8
        self.slots = SymmetricBuffer(self.points * self.point_bytes, group, dev)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        self.version = None
        self.eps = t.rms_norm_eps

    # ---------------------------------------------------------------- weights
    @torch.no_grad()
    def refresh(self, version=None) -> None:
        """Re-slice this rank's shards from the model's full (gathered) layer weights."""
        if version is not None and version == self.version:
            return
        dec, params, r = self.model.decoder, self.model.params, self.rank
        D, nq_l, nkv_l, F_l = self.D, self.nq_l, self.nkv_l, self.F_l
        q0, k0, v0 = r * nq_l * D, self.nq * D + r * nkv_l * D, (self.nq + self.nkv) * D + r * nkv_l * D
        nqd, nkd = nq_l * D, nkv_l * D
        for i in range(self.L):
            w = dec._w(params, f"layer{i}")
            for dst, src in ((self.qkv_w[i], w["qkv_w"]), (self.qkv_b[i], w["qkv_b"])):
                dst[:nqd].copy_(src[q0:q0 + nqd])
                dst[nqd:nqd + nkd].copy_(src[k0:k0 + nkd])
                dst[nqd + nkd:].copy_(src[v0:v0 + nkd])
            self.o_w[i].copy_(w["o_w"][:, q0:q0 + nqd])
            self.gu_w[i].copy_(w["gu_w"][2 * r * F_l:2 * (r + 1) * F_l])
            self.down_w[i].copy_(w["down_w"][:, r * F_l:(r + 1) * F_l])
            params.release(f"layer{i}")
        self.lm_w.copy_(dec._w(params, "head")["lm_head"][self.v0:self.v1])
        params.release("head")
        self.version = version

    # ---------------------------------------------------------------- cache
    def new_cache(self, batch: int, max_len: int) -> KVCache:
        if batch > self.max_batch:
            raise ValueError(f"tensor-parallel decode was sized for {self.max_batch} rows, got {batch}")
        m = self.model
        return KVCache(self.L, batch, self.nkv_l, max_len, self.D, m.dtype, m.device)

    @torch.no_grad()
    def load_cache(self, full: KVCache, local: KVCache, prefix_len: int) -> None:
        """Copy this rank's kv heads (first ``prefix_len`` positions) of a full cache into the local one."""
        h0, h1 = self.rank * self.nkv_l, (self.rank + 1) * self.nkv_l
        if full.block_table is None:
            local.keys[:, :, :, :prefix_len].copy_(full.keys[:, :, h0:h1, :prefix_len])
            local.values[:, :, :, :prefix_len].copy_(full.values[:, :, h0:h1, :prefix_len])
        else:   # a paged full cache: gather its rows layer by layer
            for i in range(self.L):
                k, v = full.rows(i)
                local.keys[i, :, :, :prefix_len].copy_(k[:, h0:h1, :prefix_len])
                local.values[i, :, :, :prefix_len].copy_(v[:, h0:h1, :prefix_len])
        local.lengths.copy_(full.lengths)

    # ---------------------------------------------------------------- decode
    def _reduce_norm(self, ws, meta, res, w, point: int):
        return ext().dec_residual_norm_tp(ws, list(meta), res, w, float(self.eps), self.slots.ptrs,
                                          point * self.point_bytes, self.max_batch, self.epoch.data_ptr(), self.rank)

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, cache: KVCache, rope_delta: torch.Tensor) -> torch.Tensor:
        """Logits [B, V] (identical on every rank); appends this token's local k/v and advances the cache."""
        xn = self._hidden(tokens, cache, rope_delta)
        return self.model.decoder.final_logits(self.model.params, xn, normed=True)

    @torch.no_grad()
    def decode_step_sample(self, tokens: torch.Tensor, cache: KVCache, rope_delta: torch.Tensor, *,
                           temperature: float, top_k: int, top_p: float, seed, step, row_offset: int = 0):
        """One decode step that returns the sampled (tokens, log-probs), the same on every rank.  With
        1 <= top_k <= 16 the lm_head and the sampler are vocab-parallel (no rank writes [B, V] logits);
        otherwise the replicated lm_head feeds ``ops.sample``."""
        xn = self._hidden(tokens, cache, rope_delta)
        if _FUSED_SAMPLER and 1 <= int(top_k or 0) <= ops.FUSED_SAMPLER_MAX_TOPK:
            B = xn.shape[0]
            tok = torch.empty(B, dtype=torch.int64, device=xn.device)
            lp = torch.empty(B, dtype=torch.float32, device=xn.device)
            ext().lm_head_sample_tp(xn, self.lm_w, self.v0, tok, lp, step, seed, float(temperature), int(top_k),
                                    float(top_p or 0.0), int(row_offset), self.samp_slots.ptrs, 0,
                                    self.epoch.data_ptr(), self.rank)
            return tok, lp
        logits = self.model.decoder.final_logits(self.model.params, xn, normed=True)
        return ops.sample(logits, temperature=temperature, top_k=top_k or 0, top_p=top_p or 0.0, seed=seed,
                          step=step, row_offset=row_offset)

    def _hidden(self, tokens: torch.Tensor, cache: KVCache, rope_delta: torch.Tensor) -> torch.Tensor:
        """Every decoder layer of one step; returns the final-normed hidden rows (advances the cache)."""
        m = self.model
        dec, params = m.decoder, m.params
        ext().tp_step_begin(self.epoch.data_ptr(), m.device.index if m.device.index is not None else 0)
        x = ops.embed(tokens, dec._w(params, "embed")["embed"])
        params.release("embed")
        B = tokens.shape[0]
        lens = cache.lengths
        delta = rope_delta.reshape(-1).to(torch.int64)
        lens_after = lens + 1
        w = dec._w(params, "layer0")
        xn, _ = ops.rms_norm(x, w["input_norm"], self.eps)
        for i in range(self.L):
            w = dec._w(params, f"layer{i}")
            ws, meta = ops.gemm_partials(xn, self.qkv_w[i])
            q = ops.dec_qkv(ws, meta, self.qkv_b[i], w.get("q_norm"), w.get("k_norm"), lens, delta, dec.rope,
                            cache.keys[i], cache.values[i], n_q=self.nq_l, n_kv=self.nkv_l, eps=self.eps)
            o = ops.decode_attn(q, cache.keys[i], cache.values[i], lens_after, scale=dec.scale)
            ws, meta = ops.gemm_partials(o.reshape(B, self.nq_l * self.D), self.o_w[i])
            h1, hn = self._reduce_norm(ws, meta, x, w["post_norm"], 2 * i)
            ws, meta = ops.gemm_partials(hn, self.gu_w[i])
            act = ops.dec_swiglu(ws, meta)
            ws, meta = ops.gemm_partials(act, self.down_w[i])
            nxt = dec._w(params, f"layer{i + 1}")["input_norm"] if i + 1 < self.L else dec._w(params, "head")["final_norm"]
            x, xn = self._reduce_norm(ws, meta, h1, nxt, 2 * i + 1)
            params.release(f"layer{i}")
        cache.lengths += 1
        return xn

    def close(self) -> None:
        self.slots.close()
        self.samp_slots.close()


def vocab_shard(vocab: int, world: int, rank: int, tile: int = 128):
    """Rows [v0, v1) of the lm_head that rank ``rank`` owns in the vocab-parallel sampler: contiguous shards
    of whole ``tile``-row GEMM tiles (the last one shorter), so every shard's top-k epilogue sees the same
    tiles, and column ids, as the unsharded lm_head."""
    vs = -(-vocab // (world * tile)) * tile
    return min(vocab, rank * vs), min(vocab, (rank + 1) * vs)


def tp_partition(world: int, tp_size: int):
    """Rank lists of the tensor-parallel groups: consecutive blocks of ``tp_size`` ranks (NVLink peers on one
    node), ``world // tp_size`` data-parallel replicas."""
    if tp_size < 1 or world % tp_size:
        raise ValueError(f"tp_size={tp_size} must divide the world size {world}")
    return [list(range(i, i + tp_size)) for i in range(0, world, tp_size)]


def tp_subgroup(tp_size: int):
    """This rank's tensor-parallel process group (collective: every rank creates every group, in order)."""
    world, rank = dist.get_world_size(), dist.get_rank()
    if tp_size == world:
        return None  # the default group
    mine = None
    for ranks in tp_partition(world, tp_size):
        g = dist.new_group(ranks)
        if rank in ranks:
            mine = g
    return mine


def maybe_tp_decoder(model, group=None, max_batch: int = 64) -> Optional[TPDecoder]:
    """A TPDecoder when the process group spans several GPUs with peer access, else None."""
    from vlmrl.parallel.symm import p2p_supported

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) < 2:
        return None
    if not p2p_supported(group):
        return None
    return TPDecoder(model, group, max_batch)


__all__ = ["TPDecoder", "maybe_tp_decoder", "vocab_shard", "tp_partition"]
