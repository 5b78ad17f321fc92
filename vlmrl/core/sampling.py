"""Batched KV-cache sampler (reference ``core/sampling.py:227-299``).

``Generator.generate`` runs one packed prefill over all prompts (filling the
per-sequence KV cache and sampling the first token from the prefill logits —
the reference instead discards them and re-feeds the last prompt token), then
``max_new_tokens - 1`` decode steps.  On a GPU the decode step — embedding, 36
decoder layers, lm_head, the fused top-k/top-p sampler, EOS latch and output
bookkeeping — is captured once per (batch, cache length) into a CUDA graph and
replayed, so a step is a single graph launch.  The sampler's Philox stream is
keyed by (seed, global row, step): results do not depend on how rows are
distributed over ranks.

After a row emits EOS, later positions hold EOS with log-prob 0 (the
reference's EOS latch); ``lengths`` counts tokens up to and including the first EOS.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from vlmrl import ops
from vlmrl.core.batching import pack_prompts
from vlmrl.core.types import SampleResult, SamplingConfig, VLMInputs
from vlmrl.models.qwen3vl.model import KVCache, PagedKVCache, VisionEmbeddings
from vlmrl.utils.profiling import phase


_PAGED_KV = os.environ.get("VLMRL_PAGED_KV", "1") != "0"


class _DecodeState:
    """Static buffers (and the captured graph) of one (batch, cache length) shape."""

    def __init__(self, model, B: int, max_len: int, max_new: int, num_blocks: Optional[int] = None):
        dev = model.device
        self.B, self.max_len, self.max_new = B, max_len, max_new
        self.cache = model.new_cache(B, max_len, num_blocks) if num_blocks is not None else model.new_cache(B, max_len)
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.deltas = torch.zeros(B, dtype=torch.int64, device=dev)
        self.step = torch.zeros(1, dtype=torch.int64, device=dev)
        self.seed = torch.zeros(1, dtype=torch.int64, device=dev)
        self.done = torch.zeros(B, dtype=torch.bool, device=dev)
        self.out_tok = torch.zeros(B, max_new, dtype=torch.int64, device=dev)
        self.out_lp = torch.zeros(B, max_new, dtype=torch.float32, device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.graph_cfg = None
        self.graph_kernels = 0


class Generator:
    """``tp``: a ``vlmrl.parallel.tp.TPDecoder`` — decode steps then run tensor-parallel over its ranks (every
    rank must call ``generate`` with the same prompts and seed); the prefill stays replicated."""

    def __init__(self, model, *, use_cuda_graph: bool = True, tp=None, paged_kv: Optional[bool] = None):
        self.model = model
        self.tp = tp
        # rollouts keep their KV in 64-token blocks (a group shares its prompt's blocks) unless
        # VLMRL_PAGED_KV=0 or paged_kv=False asks for one contiguous row per sequence
        self.paged_kv = _PAGED_KV if paged_kv is None else bool(paged_kv)
        self.use_cuda_graph = bool(use_cuda_graph) and model.device.type == "cuda"
        self._states: Dict[Tuple[int, int, int], _DecodeState] = {}
        self.graph_kernel_launches = 0   # kernels executed by graph replays (not seen by the launch counter)
        self.last_decode_ms = 0.0
        self.last_decode_tokens = 0

    # ---------------------------------------------------------------- one step
    def _record(self, st: _DecodeState, nt: torch.Tensor, lp: torch.Tensor, eos: Optional[int]):
        if eos is not None:
            nt = torch.where(st.done, torch.full_like(nt, eos), nt)
            lp = torch.where(st.done, torch.zeros_like(lp), lp)
            st.done |= nt == eos
        st.out_tok.index_copy_(1, st.step, nt[:, None])
        st.out_lp.index_copy_(1, st.step, lp[:, None])
        st.tok.copy_(nt)
        st.step += 1

    def _decode_step(self, st: _DecodeState, cfg: SamplingConfig, row_offset: int):
        if self.tp is None and hasattr(self.model, "decode_step_sample"):
            # lm_head + sampler fused where supported: the [B, V] logits are never written
            nt, lp = self.model.decode_step_sample(st.tok, st.cache, st.deltas, temperature=cfg.temperature,
                                                   top_k=cfg.top_k or 0, top_p=cfg.top_p or 0.0, seed=st.seed,
                                                   step=st.step, row_offset=row_offset)
            self._record(st, nt, lp, cfg.eos_id)
            return
        if self.tp is not None:
            # every rank draws the same token (vocab-parallel lm_head + sampler, or replicated logits)
            nt, lp = self.tp.decode_step_sample(st.tok, st.tp_cache, st.deltas, temperature=cfg.temperature,
                                                top_k=cfg.top_k or 0, top_p=cfg.top_p or 0.0, seed=st.seed,
                                                step=st.step, row_offset=row_offset)
            self._record(st, nt, lp, cfg.eos_id)
            return
        else:
            logits = self.model.decode_step(st.tok, st.cache, st.deltas)
        nt, lp = ops.sample(logits, temperature=cfg.temperature, top_k=cfg.top_k or 0, top_p=cfg.top_p or 0.0,
                            seed=st.seed, step=st.step, row_offset=row_offset)
        self._record(st, nt, lp, cfg.eos_id)

    def decode_time_ms(self) -> float:
        """Device time of the last generate's decode replays (synchronises on its end event)."""
        ev = getattr(self, "_pending_decode", None)
        if ev is not None:
            ev[1].synchronize()
            self.last_decode_ms = ev[0].elapsed_time(ev[1])
            self._pending_decode = None
        return self.last_decode_ms

    def _state(self, B: int, max_len: int, max_new: int, num_blocks: Optional[int] = None) -> _DecodeState:
        key = (B, max_len, max_new, num_blocks)
        st = self._states.get(key)
        if st is None:
            if len(self._states) >= 4:          # bound resident caches
                self._states.clear()
            st = _DecodeState(self.model, B, max_len, max_new, num_blocks)
            st.tp_cache = self.tp.new_cache(B, max_len) if self.tp is not None else None
            self._states[key] = st
        return st

    # ---------------------------------------------------------------- public
    @torch.no_grad()
    def generate(self, prompts: Sequence[np.ndarray], grids_per_seq, vision: Optional[VisionEmbeddings],
                 cfg: SamplingConfig, *, seed: int, row_offset: int = 0, group_size: int = 1) -> SampleResult:
        """Sample ``group_size`` continuations of every prompt; rows are ordered (prompt, member).

        Each distinct prompt is prefilled once; its KV cache rows and last-token
        logits are replicated to the other members of its group.
        """
        m = self.model
        G = len(prompts)
        gs = max(1, int(group_size))
        B = G * gs
        max_new = int(cfg.max_new_tokens)
        if cfg.temperature <= 0:
            raise ValueError("temperature must be positive")
        if B == 0 or max_new <= 0:
            empty = torch.zeros(B, 0, dtype=torch.int64)
            return SampleResult(tokens=empty, logprobs=empty.float(), lengths=torch.zeros(B, dtype=torch.int64))
        plen = max(len(p) for p in prompts)
        refeed = bool(getattr(cfg, "compat_refeed_last_token", False))
        max_len = int(-(-(plen + max_new + int(refeed)) // 64) * 64)
        paged = self.paged_kv
        nb = None
        if paged:
            # pool sized for this call's prompts, rounded up so that similar batches reuse the state
            nb = PagedKVCache.blocks_needed([len(p) for p in prompts], gs, max_len)
            nb = -(-nb // 64) * 64
        st = self._state(B, max_len, max_new, nb)
        if paged:
            st.cache.assign([len(p) for p in prompts], gs)
        batch, deltas = pack_prompts(m.spec, prompts, grids_per_seq, vision, device=m.device)
        st.cache.lengths.zero_()
        st.done.zero_()
        st.step.zero_()
        st.out_tok.zero_()
        st.out_lp.zero_()
        st.deltas.copy_(torch.from_numpy(np.repeat(deltas, gs)))
        st.seed.fill_(int(seed) & ((1 << 63) - 1))
        with phase("prefill"):
            logits = m.prefill(batch, st.cache, torch.arange(G, device=m.device) * gs)
        if gs > 1:
            if paged:
                # members already point at the leader's full prompt blocks; copy the partial last one
                st.cache.copy_prompt_tails()
            else:
                L = st.cache.keys.shape[0]
                for buf in (st.cache.keys, st.cache.values):
                    v = buf.view(L, G, gs, *buf.shape[2:])
                    v[:, :, 1:, :, :plen] = v[:, :, :1, :, :plen]
            lv = st.cache.lengths.view(G, gs)
            lv[:, 1:] = lv[:, :1]
            logits = logits.repeat_interleave(gs, dim=0)
        if not paged:
            # members' prompt KV rows are copies of their leader's: decode attention reads the leader's
            st.cache.lead.copy_(torch.arange(B, device=m.device, dtype=torch.int32) // gs * gs)
            st.cache.share_len.copy_(st.cache.lengths)
        if refeed:
            # reference start: discard the prefill logits, decode the last prompt token once more
            last = torch.tensor([int(p[-1]) for p in prompts], dtype=torch.int64).repeat_interleave(gs)
            st.tok.copy_(last.to(st.tok.device))
            logits = m.decode_step(st.tok, st.cache, st.deltas)
        nt, lp = ops.sample(logits, temperature=cfg.temperature, top_k=cfg.top_k or 0, top_p=cfg.top_p or 0.0,
                            seed=st.seed, step=st.step, row_offset=row_offset)
        self._record(st, nt, lp, cfg.eos_id)
        if self.tp is not None:
            self.tp.refresh(getattr(m.params, "version", None))
            self.tp.load_cache(st.cache, st.tp_cache, plen + int(refeed))
        steps = max_new - 1
        if steps > 0:
            if self.use_cuda_graph:
                gkey = (float(cfg.temperature), cfg.top_k, cfg.top_p, cfg.eos_id, int(row_offset),
                        getattr(m.params, "graph_epoch", 0))
                if st.graph is None or st.graph_cfg != gkey:
                    self._capture(st, cfg, row_offset)
                    st.graph_cfg = gkey
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record()
                with phase("decode"):
                    for _ in range(steps):
                        st.graph.replay()
                ev1.record()
                self._pending_decode = (ev0, ev1)
                self.graph_kernel_launches += steps * st.graph_kernels
                self.last_decode_tokens = B * steps
            else:
                for _ in range(steps):
                    self._decode_step(st, cfg, row_offset)
        toks = st.out_tok.clone()
        lps = st.out_lp.clone()
        if cfg.eos_id is not None:
            is_eos = toks == cfg.eos_id
            first = torch.where(is_eos.any(1), is_eos.float().argmax(1) + 1, torch.full_like(toks[:, 0], max_new))
        else:
            first = torch.full((B,), max_new, dtype=torch.int64, device=toks.device)
        return SampleResult(tokens=toks, logprobs=lps, lengths=first)

    def _capture(self, st: _DecodeState, cfg: SamplingConfig, row_offset: int):
        """Warm up once on a side stream, capture one decode step, then restore the mutable state.

        The warm-up writes k/v at the current cache position; the first replay
        rewrites that same position, so the cache itself needs no snapshot.
        """
        state = (st.tok, st.step, st.seed, st.done, st.out_tok, st.out_lp, st.cache.lengths)
        snap = [t.clone() for t in state]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._decode_step(st, cfg, row_offset)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        n0 = ops.launch_count()
        with ops.static_weights(), torch.cuda.graph(g):
            self._decode_step(st, cfg, row_offset)
        st.graph_kernels = ops.launch_count() - n0
        for t, v in zip(state, snap):
            t.copy_(v)
        st.graph = g


def _generator(model) -> Generator:
    gen = getattr(model, "_generator", None)
    if gen is None:
        gen = Generator(model)
        model._generator = gen
    return gen


def sample(model, params, inputs: Union[VLMInputs, torch.Tensor, np.ndarray], cfg: SamplingConfig, rng: int, *,
           tokenizer=None, return_logprobs: bool = False, row_offset: int = 0) -> SampleResult:
    """Reference-compatible entry point: ``rng`` is an integer seed (see ``vlmrl.utils.rng.RngSeq``).

    ``params`` is accepted for API compatibility; the model's own parameters are used.  ``row_offset``: the
    global index of the first row, so a batch split over data-parallel ranks draws what one process
    drawing the whole batch would (the sampler's random stream is keyed by (seed, row, step)).
    """
    if isinstance(inputs, VLMInputs):
        prompts = inputs.prompt_tokens
        if torch.is_tensor(prompts):
            prompts = [row[row != cfg.pad_id].cpu().numpy() for row in prompts]
        grids = inputs.grid_thw
        vision = inputs.vision
    else:
        arr = inputs.cpu().numpy() if torch.is_tensor(inputs) else np.asarray(inputs)
        prompts = [row[row != cfg.pad_id] for row in np.atleast_2d(arr)]
        grids = [[] for _ in prompts]
        vision = None
    res = _generator(model).generate(prompts, grids, vision, cfg, seed=int(rng), row_offset=int(row_offset))
    if tokenizer is not None:
        lens = res.lengths.tolist()
        res.texts = [tokenizer.decode(row[:n].tolist(), skip_special_tokens=True) for row, n in zip(res.tokens.cpu(), lens)]
    if not return_logprobs:
        res.logprobs = res.logprobs if res.logprobs is not None else None
    return res


__all__ = ["Generator", "sample"]
