"""CPU model tests: HF parity of the executor and hand-written backward vs autograd."""

import numpy as np
import pytest
import torch

from tests.helpers import tiny_episodes, tiny_model
from vlmrl.models.qwen3vl.api import Qwen3VLModel
from vlmrl.models.qwen3vl.model import LocalParams


def test_hf_parity_tiny():
    transformers = pytest.importorskip("transformers")
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration

    from vlmrl.models.qwen3vl.config import spec_to_config
    from vlmrl.models.qwen3vl.weights import units_to_hf_state_dict
    from vlmrl.utils.vlm import preprocess_image

    spec, units, m = tiny_model(seed=3)
    cfgd = spec_to_config(spec)
    cfgd["text_config"]["max_position_embeddings"] = 4096
    cfg = Qwen3VLConfig(**cfgd)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    hf = Qwen3VLForConditionalGeneration(cfg).eval()
    missing, unexpected = hf.load_state_dict(units_to_hf_state_dict(spec, units), strict=False)
    assert not missing and not unexpected
    rng = np.random.default_rng(0)
    pix, grid = preprocess_image(rng.integers(0, 256, (64, 96, 3), dtype=np.uint8), patch_size=16,
                                 spatial_merge_size=2, temporal_patch_size=2)
    vis = m.encode_vision(pix, grid)
    n_img = int(grid[0, 1] * grid[0, 2] // 4)
    ids = [spec.vision_start_token_id] + [spec.image_token_id] * n_img + [spec.vision_end_token_id]
    ids += list(rng.integers(0, 900, 9))
    tok = torch.tensor([ids])
    with torch.no_grad():
        hv = hf.model.visual(pix, grid_thw=grid)
        out = hf(input_ids=tok, pixel_values=pix, image_grid_thw=grid,
                 mm_token_type_ids=(tok == spec.image_token_id).long())
    torch.testing.assert_close(vis.tokens, hv.pooler_output, atol=2e-5, rtol=1e-4)
    for a, b in zip(vis.deepstack, hv.deepstack_features):
        torch.testing.assert_close(a, b, atol=2e-5, rtol=1e-4)
    logits = m.forward_vlm(tok, vis, grid)
    torch.testing.assert_close(logits, out.logits, atol=2e-5, rtol=1e-4)


def test_manual_backward_matches_autograd():
    spec, units, m = tiny_model(seed=5)
    batch, counts, _, _ = tiny_episodes(spec, m, n=3)
    M = int(batch.loss_rows.numel())
    g_lp = torch.randn(M, generator=torch.Generator().manual_seed(1))
    g_ent = torch.randn(M, generator=torch.Generator().manual_seed(2)) * 0.3

    # manual
    m.params.zero_grads()
    with torch.no_grad():
        logp, ent, ctx = m.token_logprobs(batch, save=True)
        m.backward(ctx, g_lp, g_ent)
    manual = {k: v.clone() for k, v in m.params.grads.items()}

    # autograd through the fp32 reference ops
    leaves = {k: v.detach().clone().requires_grad_(k != "visual") for k, v in units.items()}
    m2 = Qwen3VLModel(spec, params=LocalParams(leaves), dtype=torch.float32)
    logp2, ent2, _ = m2.token_logprobs(batch, save=False)
    torch.testing.assert_close(logp, logp2.detach(), atol=1e-5, rtol=1e-5)
    (g_lp * logp2 + g_ent * ent2).sum().backward()
    for name, g in manual.items():
        ref = leaves[name].grad
        assert ref is not None, name
        torch.testing.assert_close(g, ref, atol=2e-5, rtol=2e-4, msg=lambda s: f"{name}: {s}")


def test_prefill_decode_matches_full_forward():
    spec, units, m = tiny_model(seed=7)
    from vlmrl.core.batching import pack_prompts

    rng = np.random.default_rng(4)
    batch, counts, seqs, plens = tiny_episodes(spec, m, n=2, prompt_text=8, action=3)
    # prefill on the prompts, then decode the action tokens one by one; compare with full-forward logits
    prompts = [s[:p] for s, p in zip(seqs, plens)]
    grids = [[(1, 4, 4)] for _ in prompts]
    vis = batch.vision
    pb, deltas = pack_prompts(spec, prompts, grids, vis)
    cache = m.new_cache(2, 64)
    logits0 = m.prefill(pb, cache, torch.arange(2))
    full = [m.forward_vlm(torch.tensor([s]), vis.select(torch.arange(4 * i, 4 * i + 4)), [(1, 4, 4)])[0]
            for i, s in enumerate(seqs)]
    for b in range(2):
        torch.testing.assert_close(logits0[b], full[b][plens[b] - 1], atol=1e-4, rtol=1e-4)
    steps = min(len(s) - p for s, p in zip(seqs, plens)) - 1
    for t in range(steps):
        tok = torch.tensor([int(seqs[b][plens[b] + t]) for b in range(2)])
        lg = m.decode_step(tok, cache, torch.from_numpy(deltas))
        for b in range(2):
            torch.testing.assert_close(lg[b], full[b][plens[b] + t], atol=1e-4, rtol=1e-4)


def test_shared_prompt_packing_matches_full_sequences():
    """pack_groups (prompt once per group) gives the same log-probs and gradients as packing every member."""
    from vlmrl.core.batching import pack_groups, pack_sequences
    from vlmrl.utils.vlm import preprocess_image

    spec, units, m = tiny_model(seed=9)
    rng = np.random.default_rng(3)
    prompts, actions, grids, pix = [], [], [], []
    for g in range(2):
        p, gr = preprocess_image(rng.integers(0, 256, (64, 64, 3), dtype=np.uint8), patch_size=16,
                                 spatial_merge_size=2, temporal_patch_size=2)
        pix.append(p)
        grids.append([tuple(gr[0].tolist())])
        prompt = [spec.vision_start_token_id] + [spec.image_token_id] * 4 + [spec.vision_end_token_id]
        prompt += list(rng.integers(0, 900, 5 + g))
        prompts.append(np.asarray(prompt))
        actions.append([rng.integers(0, 900, n) for n in ((3, 1, 6) if g == 0 else (4, 2, 5))])
    vis = m.encode_vision(torch.cat(pix), [gg[0] for gg in grids])
    shared, c1 = pack_groups(spec, prompts, actions, grids, vis)
    seqs, plens, sgrids, rows = [], [], [], []
    for g, (p, acts) in enumerate(zip(prompts, actions)):
        for a in acts:
            seqs.append(np.concatenate([p, a]))
            plens.append(len(p))
            sgrids.append(grids[g])
            rows.append(torch.arange(4 * g, 4 * g + 4))
    full, c2 = pack_sequences(spec, seqs, plens, sgrids, vis.select(torch.cat(rows)))
    assert list(c1) == list(c2)
    assert shared.tokens.numel() < full.tokens.numel()
    M = int(full.loss_rows.numel())
    g_lp = torch.randn(M, generator=torch.Generator().manual_seed(1))
    g_ent = torch.randn(M, generator=torch.Generator().manual_seed(2)) * 0.3
    out = []
    for batch in (shared, full):
        m.params.zero_grads()
        with torch.no_grad():
            logp, ent, ctx = m.token_logprobs(batch, save=True)
            m.backward(ctx, g_lp, g_ent)
        out.append((logp.clone(), ent.clone(), {k: v.clone() for k, v in m.params.grads.items()}))
    torch.testing.assert_close(out[0][0], out[1][0], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(out[0][1], out[1][1], atol=1e-5, rtol=1e-5)
    for name in out[1][2]:
        torch.testing.assert_close(out[0][2][name], out[1][2][name], atol=2e-5, rtol=2e-4,
                                   msg=lambda s: f"{name}: {s}")


def test_qwen25_hf_parity_tiny():
    """Qwen2.5-VL family (no q/k norm, chunked MRoPE, windowed RMSNorm/SwiGLU ViT) vs HF transformers."""
    pytest.importorskip("transformers")
    from transformers import Qwen2_5_VLConfig, Qwen2_5_VLForConditionalGeneration

    from vlmrl.models.qwen25vl import get_rope_index, spec_to_config, units_to_hf_state_dict
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import init_params
    from vlmrl.utils.vlm import preprocess_image

    spec = get_preset("tiny_qwen25")
    units = init_params(spec, seed=4)
    for name, u in units.items():   # non-trivial norms and biases
        u.add_(torch.randn(u.shape, generator=torch.Generator().manual_seed(len(name))) * 0.02)
    m = Qwen3VLModel(spec, units=units, dtype=torch.float32)
    cfgd = spec_to_config(spec)
    cfgd["text_config"]["max_position_embeddings"] = 4096
    cfgd["tie_word_embeddings"] = cfgd["text_config"]["tie_word_embeddings"] = False  # lm_head was perturbed
    cfg = Qwen2_5_VLConfig(**cfgd)
    cfg._attn_implementation = "eager"
    cfg.vision_config._attn_implementation = "eager"
    cfg.text_config._attn_implementation = "eager"
    hf = Qwen2_5_VLForConditionalGeneration(cfg).eval()
    missing, unexpected = hf.load_state_dict(units_to_hf_state_dict(spec, units), strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    rng = np.random.default_rng(0)
    # 112 x 168 px -> grid (1, 8, 12): 2x3 windows of 56 px (window 4x4 patches), one partial
    pix, grid = preprocess_image(rng.integers(0, 256, (112, 168, 3), dtype=np.uint8), patch_size=14,
                                 spatial_merge_size=2, temporal_patch_size=2, min_pixels=56 * 56)
    vis = m.encode_vision(pix, grid)
    with torch.no_grad():
        hv = hf.model.visual(pix, grid_thw=grid)
    hv = getattr(hv, "pooler_output", hv)
    torch.testing.assert_close(vis.tokens, hv, atol=2e-5, rtol=1e-4)
    n_img = int(grid[0, 1] * grid[0, 2] // 4)
    ids = [spec.vision_start_token_id] + [spec.image_token_id] * n_img + [spec.vision_end_token_id]
    ids += list(rng.integers(0, 900, 9))
    pos, _ = get_rope_index(ids, [tuple(grid[0].tolist())], spatial_merge_size=2, image_token_id=spec.image_token_id)
    tok = torch.tensor([ids])
    # image frames take temporal index 0 (reference models/qwen25vl/model.py:245,283-289), rows/cols follow
    # the merged grid, text resumes at max + 1
    img = slice(1, 1 + n_img)
    assert (pos[0, img] == 1).all() and pos[1, img].max() == 1 + 3 and pos[2, img].max() == 1 + 5
    assert pos[0, 1 + n_img] == 1 + 6
    with torch.no_grad():
        mm = (tok == spec.image_token_id).int()
        # the network is compared under identical position ids
        out = hf(input_ids=tok, pixel_values=pix, image_grid_thw=grid, mm_token_type_ids=mm,
                 position_ids=torch.from_numpy(pos)[:, None, :])
    logits = m.forward_vlm(tok, vis, grid)
    torch.testing.assert_close(logits, out.logits, atol=2e-5, rtol=1e-4)


def test_compat_refeed_last_token_matches_duplicated_prompt():
    """``compat_refeed_last_token``: the first token comes from decoding the last prompt token again."""
    from vlmrl.core.sampling import Generator
    from vlmrl.core.types import SamplingConfig

    spec, units, m = tiny_model(seed=4)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(1, 900, 7), rng.integers(1, 900, 11)]
    gen = Generator(m)
    for refeed in (False, True):
        cfg = SamplingConfig(temperature=1.0, top_k=1, max_new_tokens=3, compat_refeed_last_token=refeed)
        res = gen.generate(prompts, [[], []], None, cfg, seed=3)
        for i, p in enumerate(prompts):
            seq = list(p) + ([int(p[-1])] if refeed else [])
            for t in range(3):
                logits = m.forward_text(torch.tensor([seq]))[0, -1]
                want = int(logits.argmax())
                assert int(res.tokens[i, t]) == want, (refeed, i, t)
                seq.append(want)


def test_decay_frozen_matches_reference_drift():
    """``AdamWConfig.decay_frozen``: the frozen vision tower shrinks by (1 - lr*wd) per step, in fp32."""
    from vlmrl.core.optim import AdamWConfig, LocalOptimizer

    spec, units, m = tiny_model(seed=2)
    assert "visual" in m.params.units and "visual" not in m.params.trainable
    v0 = m.params.units["visual"].clone()
    lr, wd = 1e-3, 0.5
    for decay in (False, True):
        m.params.units["visual"].copy_(v0)
        opt = LocalOptimizer(m.params, AdamWConfig(lr=lr, weight_decay=wd, decay_frozen=decay))
        for step in range(1, 4):
            opt.step(step)
        want = v0 * (1 - lr * wd) ** 3 if decay else v0
        torch.testing.assert_close(m.params.units["visual"], want, rtol=1e-6, atol=1e-7)
        torch.testing.assert_close(opt.all_param_units()["visual"], want, rtol=1e-6, atol=1e-7)
