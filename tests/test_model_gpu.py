"""Tiny Qwen3-VL on the GPU (bf16, native kernels) against the fp32 CPU executor."""

import numpy as np
import pytest
import torch

from tests.helpers import tiny_episodes, tiny_model
from vlmrl.models.qwen3vl.api import Qwen3VLModel

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_tiny_forward_backward_gpu_vs_cpu():
    spec, units, m_cpu = tiny_model(seed=11)
    m_gpu = Qwen3VLModel(spec, units=units, dtype=torch.bfloat16, device="cuda")
    b_cpu, _, _, _ = tiny_episodes(spec, m_cpu, n=4)
    b_gpu, _, _, _ = tiny_episodes(spec, m_gpu, n=4, device="cuda")
    lp_c, ent_c, ctx_c = m_cpu.token_logprobs(b_cpu, save=True)
    lp_g, ent_g, ctx_g = m_gpu.token_logprobs(b_gpu, save=True)
    assert (lp_g.cpu() - lp_c).abs().max().item() < 0.1
    assert (ent_g.cpu() - ent_c).abs().max().item() < 0.1
    M = lp_c.numel()
    g1 = torch.randn(M, generator=torch.Generator().manual_seed(0))
    g2 = torch.randn(M, generator=torch.Generator().manual_seed(1)) * 0.1
    m_cpu.params.zero_grads()
    m_gpu.params.zero_grads()
    with torch.no_grad():
        m_cpu.backward(ctx_c, g1, g2)
        m_gpu.backward(ctx_g, g1.cuda(), g2.cuda())
    for name, g in m_cpu.params.grads.items():
        assert _rel(m_gpu.params.grads[name].cpu(), g) < 0.08, name
    from vlmrl.ops._ext import ext

    assert ext().read_and_clear_error(torch.cuda.current_device()) == 0


def test_tiny_prefill_decode_gpu():
    from vlmrl.core.batching import pack_prompts

    spec, units, _ = tiny_model(seed=13)
    m = Qwen3VLModel(spec, units=units, dtype=torch.bfloat16, device="cuda")
    batch, _, seqs, plens = tiny_episodes(spec, m, n=3, prompt_text=9, action=4, device="cuda")
    prompts = [s[:p] for s, p in zip(seqs, plens)]
    pb, deltas = pack_prompts(spec, prompts, [[(1, 4, 4)]] * 3, batch.vision, device="cuda")
    cache = m.new_cache(3, 64)
    lg = m.prefill(pb, cache, torch.arange(3, device="cuda"))
    for b in range(3):
        vis = batch.vision.select(torch.arange(4 * b, 4 * b + 4, device="cuda"))
        full = m.forward_vlm(torch.tensor([seqs[b]]), vis, [(1, 4, 4)])[0]
        assert (lg[b] - full[plens[b] - 1]).abs().max().item() < 0.05
        tok = torch.tensor([int(seqs[i][plens[i]]) for i in range(3)], device="cuda")
    step = m.decode_step(tok, cache, torch.from_numpy(deltas).cuda())
    for b in range(3):
        vis = batch.vision.select(torch.arange(4 * b, 4 * b + 4, device="cuda"))
        full = m.forward_vlm(torch.tensor([seqs[b]]), vis, [(1, 4, 4)])[0]
        assert (step[b] - full[plens[b]]).abs().max().item() < 0.05
