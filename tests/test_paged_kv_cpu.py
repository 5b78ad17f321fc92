"""Paged KV cache on the CPU executor: block-table layout, prompt-block sharing inside a GRPO group, and
rollouts that match the contiguous cache token for token."""

import numpy as np
import torch

from vlmrl import ops
from vlmrl.core.sampling import Generator
from vlmrl.core.types import SamplingConfig
from vlmrl.models.qwen3vl.api import Qwen3VLModel
from vlmrl.models.qwen3vl.config import get_preset
from vlmrl.models.qwen3vl.model import PagedKVCache


def test_assign_shares_full_prompt_blocks_and_owns_the_rest():
    c = PagedKVCache(2, 6, 2, 256, 8, num_blocks=64, dtype=torch.float32)
    used = c.assign([130, 64], group_size=3)       # prompt 0: 2 full blocks + a partial; prompt 1: 1 full
    assert used == PagedKVCache.blocks_needed([130, 64], 3, 256) == (2 + 3 * 2) + (1 + 3 * 3)
    t = c.block_table.numpy()
    # members of a group name the leader's full prompt blocks, nothing else is shared
    assert (t[0, :2] == t[1, :2]).all() and (t[0, :2] == t[2, :2]).all()
    assert (t[3, :1] == t[4, :1]).all() and (t[3, :1] == t[5, :1]).all()
    own = np.concatenate([t[0, 2:], t[1, 2:], t[2, 2:], t[3, 1:], t[4, 1:], t[5, 1:], t[0, :2], t[3, :1]])
    assert len(set(own.tolist())) == own.size and own.max() < used
    # the partial prompt block (prompt 0, block 2) is copied leader -> members after the prefill
    c.keys[:, t[0, 2]] = 7.0
    c.copy_prompt_tails()
    assert (c.keys[:, t[1, 2]] == 7.0).all() and (c.keys[:, t[2, 2]] == 7.0).all()
    assert (c.keys[:, t[4, 1]] == 0).all()         # prompt 1 ends on a block boundary: nothing to copy


def test_paged_write_and_attention_match_contiguous():
    g = torch.Generator().manual_seed(0)
    B, Hkv, Hq, D, T = 3, 2, 4, 16, 192
    paged = PagedKVCache(1, B, Hkv, T, D, num_blocks=16, dtype=torch.float32)
    paged.assign([70, 10, 150], group_size=1)
    k = torch.randn(B * T, Hkv, D, generator=g)
    v = torch.randn(B * T, Hkv, D, generator=g)
    seq = torch.arange(B).repeat_interleave(T)
    pos = torch.arange(T).repeat(B)
    dense_k = torch.zeros(B, Hkv, T, D)
    dense_v = torch.zeros(B, Hkv, T, D)
    ops.kv_write(k, v, dense_k, dense_v, seq, pos)
    ops.kv_write(k, v, paged.keys[0], paged.values[0], seq, pos, paged.block_table)
    pk, pv = paged.rows(0)
    assert torch.equal(pk, dense_k) and torch.equal(pv, dense_v)
    q = torch.randn(B, Hq, D, generator=g)
    lens = torch.tensor([70, 1, 150], dtype=torch.int32)
    a = ops.decode_attn(q, dense_k, dense_v, lens)
    b = ops.decode_attn(q, paged.keys[0], paged.values[0], lens, block_table=paged.block_table)
    torch.testing.assert_close(a, b)


def test_grouped_rollout_paged_equals_contiguous():
    spec = get_preset("tiny")
    m = Qwen3VLModel(spec, dtype=torch.float32, seed=1)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 900, n) for n in (70, 9, 64)]
    cfg = SamplingConfig(temperature=0.8, top_k=20, top_p=0.95, eos_id=None, pad_id=0, max_new_tokens=12)
    out = []
    for paged in (False, True):
        gen = Generator(m, paged_kv=paged)
        res = gen.generate(prompts, [[]] * 3, None, cfg, seed=5, group_size=4)
        out.append(res)
        st = next(iter(gen._states.values()))
        assert (st.cache.block_table is not None) == paged
    assert torch.equal(out[0].tokens, out[1].tokens)
    torch.testing.assert_close(out[0].logprobs, out[1].logprobs)
