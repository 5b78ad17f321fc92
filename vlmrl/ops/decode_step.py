"""Host side of the persistent decode step (``csrc/decode_step.cu``).

One cooperative launch runs every decoder layer of a decode step: the weight stream of all four GEMMs of
all layers is walked by a TMA producer warp per SM that never waits on activations, so HBM keeps
streaming while the CTA computes attention or a norm.  ``DecodeStepPlan`` owns what that launch reads:
the tensor maps of every weight matrix and of the four activation buffers, a per-layer pointer table
(bias, norms, cache slices), the activation and partial-sum buffers and the arrival counters.  A plan is
bound to one parameter set (addresses), one KV cache and one batch size; the decode CUDA graph keeps it
alive, so every replay reuses the same buffers.

Reference: the decode loop ``core/sampling.py:157-224`` (one jitted step per generated token).
"""

from __future__ import annotations

import os
from typing import List

import torch

from vlmrl.ops._ext import ext

# VLMRL_DECODE_PERSISTENT=1 selects the persistent step.  Off by default: it is correct (bitwise
# reproducible, tested against the per-kernel path) but measured slower on the 4B model at batch 64
# (6.8 vs 4.1 ms per step): its GEMM phases run at about a quarter of the HBM rate.
ENABLED = os.environ.get("VLMRL_DECODE_PERSISTENT", "0") == "1"

_MAX_BATCH = 128


def supported(spec_text, batch: int) -> bool:
    """Shapes the persistent kernel handles: head_dim 128, GQA ratio 1/2/4/8, batch <= 128, hidden <= 4096
    and a multiple of 128, intermediate a multiple of 64.  (The tensor maps of the cached prefix and the
    plan are bound to the cache buffers, so the cache must stay at its address while a plan exists.)"""
    t = spec_text
    nq, nkv = t.num_attention_heads, t.num_key_value_heads
    return (t.head_dim == 128 and nq % nkv == 0 and (nq // nkv) in (1, 2, 4, 8) and 1 <= batch <= _MAX_BATCH
            and t.hidden_size % 128 == 0 and t.hidden_size <= 4096 and t.intermediate_size % 64 == 0)


class DecodeStepPlan:
    """Tables and buffers of the persistent decode step for (weights, cache, batch)."""

    def __init__(self, decoder, params, cache, batch: int):
        t = decoder.spec.text
        dev = cache.keys.device
        self.B = int(batch)
        self.L, self.H = t.num_hidden_layers, t.hidden_size
        self.nq, self.nkv, self.F = t.num_attention_heads, t.num_key_value_heads, t.intermediate_size
        self.D = t.head_dim
        self.Tmax = int(cache.keys.shape[3])
        self.eps, self.scale = float(decoder.eps), float(decoder.scale)
        B, H, F = self.B, self.H, self.F
        bf = torch.bfloat16
        self.x = torch.empty(B, H, dtype=bf, device=dev)
        self.h1 = torch.empty(B, H, dtype=bf, device=dev)
        self.xn = torch.empty(B, H, dtype=bf, device=dev)
        self.o = torch.empty(B, self.nq * self.D, dtype=bf, device=dev)
        self.hn = torch.empty(B, H, dtype=bf, device=dev)
        self.act = torch.empty(B, F, dtype=bf, device=dev)
        self.dims = [self.L, B, H, self.nq, self.nkv, F, self.Tmax]
        grid = torch.cuda.get_device_properties(dev).multi_processor_count
        self.ws = torch.empty(int(ext().decode_step_ws_floats(self.dims, grid)), dtype=torch.float32, device=dev)
        self.ssq = torch.empty(2 * B * (H // 128), dtype=torch.float32, device=dev)
        self.sync = torch.zeros(int(ext().decode_step_sync_words(self.L, F, B)), dtype=torch.int32, device=dev)
        weights: List[torch.Tensor] = []
        rows: List[List[int]] = []
        self._keep: List[torch.Tensor] = []   # every tensor whose address the tables hold
        head = decoder._w(params, "head")
        for i in range(self.L):
            w = decoder._w(params, f"layer{i}")
            nxt = decoder._w(params, f"layer{i + 1}")["input_norm"] if i + 1 < self.L else head["final_norm"]
            mats = [w["qkv_w"], w["o_w"], w["gu_w"], w["down_w"]]
            for m in mats:
                if not (torch.is_tensor(m) and m.dtype == bf and m.is_contiguous()):
                    raise TypeError("persistent decode step needs resident bf16 weight tensors")
            weights += mats
            qn, kn = w.get("q_norm"), w.get("k_norm")
            ptrs = [w["qkv_b"].data_ptr() if w.get("qkv_b") is not None else 0,
                    qn.data_ptr() if qn is not None else 0, kn.data_ptr() if kn is not None else 0,
                    w["post_norm"].data_ptr(), nxt.data_ptr(), cache.keys[i].data_ptr(), cache.values[i].data_ptr(), 0]
            rows.append(ptrs)
            self._keep += mats + [w["post_norm"], nxt] + [v for v in (w.get("qkv_b"), qn, kn) if v is not None]
        BP = max(16, (B + 15) // 16 * 16)
        caches = []
        for i in range(self.L):
            caches += [cache.keys[i], cache.values[i]]
        wm, am = ext().decode_step_maps(weights, caches, [self.xn, self.o, self.hn, self.act], BP)
        self.wmaps = wm.to(dev)
        self.amaps = am.to(dev)
        self.layers = torch.tensor(rows, dtype=torch.int64).to(dev)
        self.cache_keys = cache.keys
        self.inv_freq = decoder.rope.device_tables(dev)[0]
        # VLMRL_DS_TRACE=1: the kernel stamps phase boundaries (globaltimer ns) into trace[:G * L * 16] as
        # [G, L, 16] and adds per-CTA wait cycles into the [G, 16] block after it
        self.trace = (torch.zeros(grid * (self.L + 1) * 16 + 4 * 256, dtype=torch.int64, device=dev)
                      if os.environ.get("VLMRL_DS_TRACE", "0") == "1" else None)

    def run(self, lens: torch.Tensor, delta: torch.Tensor, lead=None, share_len=None) -> torch.Tensor:
        """One decode step on ``self.x`` (embedded tokens) / ``self.xn`` (layer-0 input norm of them).

        Appends this step's k / v at ``lens`` in every layer's cache (lengths are not advanced) and returns
        the final-normed hidden state ``self.xn`` [B, H]."""
        ext().decode_step(self.wmaps, self.amaps, self.layers, self.x, self.h1, self.xn, self.o, self.hn, self.act,
                          self.ws, self.ssq, self.sync, lens, delta, self.inv_freq, lead, share_len, self.dims, self.eps,
                          self.scale, self.trace)
        return self.xn


def plan_for(decoder, params, cache, batch: int) -> DecodeStepPlan:
    """The plan of (decoder, parameter addresses, batch), cached on the KV cache object: a decode CUDA graph
    that captured a plan's addresses lives no longer than its cache, so the plan lives exactly as long."""
    w0 = decoder._w(params, "layer0")["qkv_w"]
    key = (id(decoder), int(batch), id(params), getattr(params, "graph_epoch", 0), w0.data_ptr())
    plans = cache.__dict__.setdefault("_decode_plans", {})
    plan = plans.get(key)
    if plan is None:
        # a new parameter epoch re-captures the decode graph, so only the newest plans can still be replayed
        while len(plans) >= 2:
            plans.pop(next(iter(plans)))
        plan = DecodeStepPlan(decoder, params, cache, batch)
        plans[key] = plan
    return plan


__all__ = ["DecodeStepPlan", "plan_for", "supported", "ENABLED"]
