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


@pytest.mark.gpu
def test_shared_prompt_training_step_matches_full_on_gpu():
    """bf16 CUDA path: log-probs and gradients of pack_groups agree with per-member packing."""
    import numpy as np

    from vlmrl.core.batching import pack_groups, pack_sequences
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import init_params
    from vlmrl.utils.vlm import preprocess_image

    spec = get_preset("tiny")
    units = init_params(spec, seed=2)
    m = Qwen3VLModel(spec, units=units, dtype=torch.bfloat16, device="cuda")
    rng = np.random.default_rng(5)
    prompts, actions, grids, pix = [], [], [], []
    for g in range(3):
        p, gr = preprocess_image(rng.integers(0, 256, (64, 64, 3), dtype=np.uint8), patch_size=16,
                                 spatial_merge_size=2, temporal_patch_size=2)
        pix.append(p)
        grids.append([tuple(gr[0].tolist())])
        prompt = [spec.vision_start_token_id] + [spec.image_token_id] * 4 + [spec.vision_end_token_id]
        prompt += list(rng.integers(0, 900, 70 + 5 * g))
        prompts.append(np.asarray(prompt))
        actions.append([rng.integers(0, 900, n) for n in (33, 1, 80, 64)])
    vis = m.encode_vision(torch.cat(pix).cuda().to(torch.bfloat16), [gg[0] for gg in grids])
    shared, c1 = pack_groups(spec, prompts, actions, grids, vis, device="cuda")
    seqs, plens, sgrids, rows = [], [], [], []
    for g, (p, acts) in enumerate(zip(prompts, actions)):
        for a in acts:
            seqs.append(np.concatenate([p, a]))
            plens.append(len(p))
            sgrids.append(grids[g])
            rows.append(torch.arange(4 * g, 4 * g + 4))
    full, c2 = pack_sequences(spec, seqs, plens, sgrids, vis.select(torch.cat(rows).cuda()), device="cuda")
    M = int(full.loss_rows.numel())
    g_lp = torch.randn(M, device="cuda")
    g_ent = torch.randn(M, device="cuda") * 0.3
    out = []
    for batch in (shared, full):
        m.params.zero_grads()
        with torch.no_grad():
            logp, ent, ctx = m.token_logprobs(batch, save=True)
            m.backward(ctx, g_lp, g_ent)
        out.append((logp.float().clone(), {k: v.clone() for k, v in m.params.grads.items()}))
    torch.testing.assert_close(out[0][0], out[1][0], atol=3e-2, rtol=3e-2)
    for name, gf in out[1][1].items():
        gs = out[0][1][name]
        rel = float((gs - gf).norm() / gf.norm().clamp_min(1e-12))
        assert rel < 3e-2, (name, rel)


def test_tiny_qwen25_gpu_vs_cpu():
    """Qwen2.5-VL family on the CUDA path: windowed ViT, rotation-only q/k, chunked MRoPE, fused decode."""
    from vlmrl.core.batching import pack_prompts
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import init_params
    from vlmrl.utils.vlm import preprocess_image

    spec = get_preset("tiny_qwen25")
    units = init_params(spec, seed=6)
    m_cpu = Qwen3VLModel(spec, units=units, dtype=torch.float32)
    m_gpu = Qwen3VLModel(spec, units=units, dtype=torch.bfloat16, device="cuda")
    rng = np.random.default_rng(1)
    pix, grid = preprocess_image(rng.integers(0, 256, (112, 168, 3), dtype=np.uint8), patch_size=14,
                                 spatial_merge_size=2, temporal_patch_size=2, min_pixels=56 * 56)
    vc = m_cpu.encode_vision(pix, grid)
    vg = m_gpu.encode_vision(pix.cuda().to(torch.bfloat16), grid)
    assert _rel(vg.tokens.cpu(), vc.tokens) < 0.03
    n_img = int(grid[0, 1] * grid[0, 2] // 4)
    ids = [spec.vision_start_token_id] + [spec.image_token_id] * n_img + [spec.vision_end_token_id]
    ids += list(rng.integers(0, 900, 12))
    g3 = [tuple(grid[0].tolist())]
    lc = m_cpu.forward_vlm(torch.tensor([ids]), vc, g3)[0]
    lg = m_gpu.forward_vlm(torch.tensor([ids]), vg, g3)[0]
    assert _rel(lg.cpu(), lc) < 0.03
    # prefill the first P tokens, then one fused decode step equals the full forward
    P = len(ids) - 3
    pb, deltas = pack_prompts(spec, [np.asarray(ids[:P])], [g3], vg, device="cuda")
    cache = m_gpu.new_cache(1, 64)
    m_gpu.prefill(pb, cache, torch.arange(1, device="cuda"))
    step = m_gpu.decode_step(torch.tensor([ids[P]], device="cuda"), cache, torch.from_numpy(deltas).cuda())
    assert (step[0].float() - lg[P].float()).abs().max().item() < 0.05


def test_reference_vision_tower_gpu_vs_cpu():
    """The reference's Qwen3-VL tower variant (RMSNorm/SwiGLU, 4-token windows, its rotary) on the CUDA path."""
    from dataclasses import replace

    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import init_params

    spec = get_preset("tiny", vision_arch="reference")
    spec = replace(spec, vision=replace(spec.vision, window_size=32, num_position_embeddings=None))
    units = init_params(spec, seed=8)
    units["visual"] += 0.05 * torch.randn(units["visual"].shape, generator=torch.Generator().manual_seed(2))
    m_cpu = Qwen3VLModel(spec, units=units, dtype=torch.float32)
    m_gpu = Qwen3VLModel(spec, units=units, dtype=torch.bfloat16, device="cuda")
    grid = [(1, 8, 12)]
    pix = torch.randn(96, spec.vision.patch_volume, generator=torch.Generator().manual_seed(4))
    vc = m_cpu.encode_vision(pix, grid)
    vg = m_gpu.encode_vision(pix.cuda().to(torch.bfloat16), grid)
    assert _rel(vg.tokens.cpu(), vc.tokens) < 0.03
    assert len(vg.deepstack) == len(vc.deepstack) == 1
    assert _rel(vg.deepstack[0].cpu(), vc.deepstack[0]) < 0.03
