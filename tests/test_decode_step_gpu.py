"""Persistent decode step (one cooperative launch for all layers) against the per-kernel decode path.

The per-kernel path (stream-K GEMMs + fused consumer kernels + decode attention) is itself checked
against the fp32 CPU executor in test_model_gpu.py.  Here both paths run one decode step from the same
cache contents; the final-normed hidden state and the k/v appended to every layer's cache must agree
within bf16 tolerance.  Cases cover GQA 4 with q/k RMSNorm (Qwen3), GQA 2 with q/k/v bias and no q/k
norm (Qwen2.5), batch sizes that pad the MMA's N dimension (5, 100) or fill it (64), ragged cache
lengths, and GRPO-style shared prompt rows (lead / share_len).
"""

import pytest
import torch

from vlmrl.ops import decode_step as _ds

from vlmrl.models.qwen3vl.api import Qwen3VLModel
from vlmrl.models.qwen3vl.config import Qwen3VLSpec, TextBackboneSpec

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _persistent_on(monkeypatch):
    """The persistent step is opt-in; these tests switch it on."""
    monkeypatch.setattr(_ds, "ENABLED", True)


def _spec(kind: str) -> Qwen3VLSpec:
    if kind == "qwen3":
        t = TextBackboneSpec(hidden_size=512, num_attention_heads=8, num_hidden_layers=3, num_key_value_heads=2,
                             head_dim=128, intermediate_size=768, rope_theta=5e6, rope_section=(24, 20, 20),
                             mrope_interleaved=True, vocab_size=1024)
    else:
        t = TextBackboneSpec(hidden_size=384, num_attention_heads=4, num_hidden_layers=2, num_key_value_heads=2,
                             head_dim=128, intermediate_size=640, rope_theta=1e6, rope_section=(16, 24, 24),
                             mrope_interleaved=False, vocab_size=1024, attention_bias=True, qk_norm=False)
    return Qwen3VLSpec(text=t, vision=None, eos_token_id=1000, pad_token_id=1001)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _randomise_biases(m: Qwen3VLModel, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    for i in range(m.spec.text.num_hidden_layers):
        w = m.decoder._w(m.params, f"layer{i}")
        for name in ("qkv_b", "q_norm", "k_norm", "input_norm", "post_norm"):
            t = w.get(name)
            if t is not None:
                base = 0.0 if name == "qkv_b" else 1.0
                t.copy_((base + 0.1 * torch.randn(t.shape, generator=g, device="cuda")).to(t.dtype))


@pytest.mark.parametrize("kind,B,share", [("qwen3", 5, False), ("qwen3", 64, True), ("qwen3", 100, False),
                                          ("qwen25", 16, True)])
def test_persistent_decode_step_matches_kernel_path(kind, B, share):
    from vlmrl.ops import decode_step
    from vlmrl.ops._ext import ext

    spec = _spec(kind)
    m = Qwen3VLModel(spec, dtype=torch.bfloat16, device="cuda", seed=3)
    _randomise_biases(m, 5)
    dec = m.decoder
    assert decode_step.supported(spec.text, B)
    Tmax = 192
    g = torch.Generator(device="cuda").manual_seed(B)
    cache = m.new_cache(B, Tmax)
    L = spec.text.num_hidden_layers
    cache.keys.copy_(torch.randn(cache.keys.shape, generator=g, device="cuda").to(torch.bfloat16))
    cache.values.copy_(torch.randn(cache.values.shape, generator=g, device="cuda").to(torch.bfloat16))
    lens = torch.randint(1, Tmax - 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    if share:
        gs = 4
        lead = (torch.arange(B, device="cuda", dtype=torch.int32) // gs) * gs
        plen = torch.randint(1, 60, (B,), generator=g, device="cuda", dtype=torch.int32)[lead.long()]
        for b in range(B):
            lb = int(lead[b])
            n = int(plen[b])
            cache.keys[:, b, :, :n] = cache.keys[:, lb, :, :n]
            cache.values[:, b, :, :n] = cache.values[:, lb, :, :n]
        lens = torch.maximum(lens, plen + 1)
        cache.lead.copy_(lead)
        cache.share_len.copy_(plen)
    cache.lengths.copy_(lens)
    # poison the slots past each row's length: neither path may read them
    for b in range(B):
        n = int(lens[b])
        cache.keys[:, b, :, n + 1:] = float("nan")
        cache.values[:, b, :, n + 1:] = float("nan")
    tokens = torch.randint(0, 1000, (B,), generator=g, device="cuda")
    delta = torch.randint(-50, 50, (B,), generator=g, device="cuda")

    ref_cache = m.new_cache(B, Tmax)
    for name in ("keys", "values", "lengths", "lead", "share_len"):
        getattr(ref_cache, name).copy_(getattr(cache, name))

    with torch.no_grad():
        assert dec._persistent_ok(m.params, B)
        h_p, normed = dec.decode_hidden(m.params, tokens, cache, delta)
        assert normed
        h_p = h_p.clone()
        torch.cuda.synchronize()
        words = ext().read_error_words(torch.cuda.current_device())
        assert words[0] == 0, f"error {words[0]} in CTA {words[1]} at sync word {words[2]} (seen {words[3]})"
        from vlmrl import ops

        e = dec._w(m.params, "embed")["embed"]
        h_k = dec._decode_fused(m.params, ops.embed(tokens, e), ref_cache, delta)
        torch.cuda.synchronize()
    assert torch.isfinite(h_p.float()).all()
    assert _rel(h_p, h_k) < 2e-2, _rel(h_p, h_k)
    rows = torch.arange(B, device="cuda")
    pos = lens.long()
    for i in range(L):
        kp = cache.keys[i][rows, :, pos]
        kk = ref_cache.keys[i][rows, :, pos]
        vp = cache.values[i][rows, :, pos]
        vk = ref_cache.values[i][rows, :, pos]
        assert _rel(kp, kk) < 2e-2 and _rel(vp, vk) < 2e-2, i
    # a second step from the advanced cache reuses the plan (same buffers and tables)
    plan_count = len(cache.__dict__["_decode_plans"])
    cache.lengths += 1
    ref_cache.lengths += 1
    with torch.no_grad():
        h_p2 = dec.decode_hidden(m.params, tokens.flip(0), cache, delta)[0].clone()
        h_k2 = dec._decode_fused(m.params, ops.embed(tokens.flip(0), e), ref_cache, delta)
    torch.cuda.synchronize()
    assert len(cache.__dict__["_decode_plans"]) == plan_count
    assert _rel(h_p2, h_k2) < 2e-2
    assert ext().read_and_clear_error(torch.cuda.current_device()) == 0


def test_persistent_decode_step_is_deterministic_and_graph_capturable():
    from vlmrl.ops._ext import ext

    spec = _spec("qwen3")
    m = Qwen3VLModel(spec, dtype=torch.bfloat16, device="cuda", seed=7)
    B, Tmax = 24, 128
    g = torch.Generator(device="cuda").manual_seed(1)
    cache = m.new_cache(B, Tmax)
    cache.keys.copy_(torch.randn(cache.keys.shape, generator=g, device="cuda").to(torch.bfloat16))
    cache.values.copy_(torch.randn(cache.values.shape, generator=g, device="cuda").to(torch.bfloat16))
    cache.lengths.copy_(torch.randint(1, 100, (B,), generator=g, device="cuda", dtype=torch.int32))
    tokens = torch.randint(0, 1000, (B,), generator=g, device="cuda")
    delta = torch.zeros(B, dtype=torch.int64, device="cuda")
    with torch.no_grad():
        a = m.decode_step(tokens, cache, delta).clone()
        cache.lengths -= 1
        b = m.decode_step(tokens, cache, delta).clone()
        cache.lengths -= 1
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                out = m.decode_step(tokens, cache, delta)
        torch.cuda.current_stream().wait_stream(s)
        graph.replay()  # capture recorded the step without running it: lengths are still those of a / b
        torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(out, a)
    assert ext().read_and_clear_error(torch.cuda.current_device()) == 0
