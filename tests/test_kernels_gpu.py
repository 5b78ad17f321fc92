"""GPU kernel tests: every CUDA op against its fp32 PyTorch oracle (vlmrl.ops.reference)."""

import math

import numpy as np

import pytest
import torch

from vlmrl import ops
from vlmrl.ops import reference as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ext_loaded():
    from vlmrl.ops._ext import ext, loaded_path

    ext()
    assert loaded_path().endswith(".so")


def _r(*shape, scale=1.0, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(dtype)


def _close(out, exp, rtol=2e-2, atol=2e-2, name=""):
    out, exp = out.float(), exp.float()
    err = (out - exp).abs().max().item()
    lim = atol + rtol * exp.abs().max().item()
    assert err <= lim, f"{name}: max err {err:.4g} > {lim:.4g}"


def _no_device_error():
    from vlmrl.ops._ext import ext

    assert ext().read_and_clear_error(torch.cuda.current_device()) == 0


def test_extension_loaded():
    _ext_loaded()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 392, 136), (1000, 2056, 520), (64, 6144, 2560), (4096, 4096, 2560)])
def test_gemm_nt(M, N, K):
    a, b = _r(M, K, seed=1), _r(N, K, seed=2)
    bias, res = _r(N, seed=3), _r(M, N, seed=4)
    out = ops.gemm(a, b)
    _close(out, ref.gemm(a, b, out_dtype=torch.float32), name="nt")
    out = ops.gemm(a, b, bias=bias, residual=res, alpha=0.5)
    _close(out, ref.gemm(a, b, bias=bias, residual=res, alpha=0.5, out_dtype=torch.float32), name="nt+epi")
    out32 = ops.gemm(a, b, out_dtype=torch.float32)
    _close(out32, ref.gemm(a, b, out_dtype=torch.float32), rtol=5e-3, atol=5e-3, name="nt f32")
    _no_device_error()


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (192, 264, 200), (2048, 2560, 9728)])
def test_gemm_nn_tn(M, N, K):
    dy = _r(M, K, seed=5)          # [M, K]
    w = _r(K, N, seed=6)           # stored [K, N] (MN-major B)
    _close(ops.gemm(dy, w, b_kmajor=False), dy.float() @ w.float(), name="nn")
    x = _r(K, N, seed=7)           # dW [M?]: A stored [K, M], B stored [K, N]
    a = _r(K, M, seed=8)
    acc = torch.ones(M, N, device=DEV, dtype=torch.float32)
    ops.gemm(a, x, a_kmajor=False, b_kmajor=False, accumulate=acc)
    _close(acc, a.float().t() @ x.float() + 1.0, rtol=5e-3, atol=5e-3, name="tn acc")
    _no_device_error()


@pytest.mark.parametrize("M,N,K", [(64, 2560, 4096), (64, 19456, 2560), (7, 160, 1024), (64, 151936, 2560), (200, 6144, 2560)])
def test_gemm_splitk_skinny(M, N, K):
    x, w = _r(M, K, seed=40), _r(N, K, scale=0.05, seed=41)
    res, b = _r(M, N, seed=42), _r(N, seed=43)
    _close(ops.gemm(x, w, bias=b, residual=res), ref.gemm(x, w, bias=b, residual=res, out_dtype=torch.float32),
           name="splitk store")
    act, pre = ops.linear_swiglu(x, w)
    pre_ref = ref.gemm(x, w, out_dtype=torch.float32)
    _close(pre, pre_ref, name="splitk swiglu pre")
    _close(act, ref.swiglu_interleaved(pre_ref.to(torch.bfloat16)), name="splitk swiglu")
    _no_device_error()


def test_gemm_activation_epilogues():
    M, N, K = 300, 512, 256
    x, w = _r(M, K, seed=9), _r(N, K, scale=0.1, seed=10)
    act, pre = ops.linear_swiglu(x, w)
    pre_ref = ref.gemm(x, w, out_dtype=torch.float32)
    _close(pre, pre_ref, name="swiglu pre")
    _close(act, ref.swiglu_interleaved(pre_ref.to(torch.bfloat16)), name="swiglu act")
    b = _r(N, seed=11)
    for epi, approx in ((ops.EPI_GELU_TANH, "tanh"), (ops.EPI_GELU_ERF, "none")):
        out = ops.gemm(x, w, bias=b, epilogue=epi)
        _close(out, ref.gelu(ref.gemm(x, w, bias=b, out_dtype=torch.float32), approx), name=f"gelu {approx}")
    _no_device_error()


def test_norms():
    x, w = _r(333, 2560, seed=12), (1 + 0.1 * _r(2560, seed=13).float()).to(torch.bfloat16)
    y, r = ops.rms_norm(x, w, 1e-6)
    yr, rr = ref.rms_norm(x, w, 1e-6)
    _close(y, yr, name="rms")
    _close(r, rr, rtol=1e-4, atol=1e-5, name="rstd")
    dy = _r(333, 2560, seed=14)
    dw = torch.zeros(2560, device=DEV)
    dx = ops.rms_norm_bwd(dy, x, w, r, dw_accum=dw)
    dxr, dwr = ref.rms_norm_bwd(dy, x, w, rr)
    _close(dx, dxr, name="rms dx")
    _close(dw, dwr, rtol=1e-3, atol=1e-3, name="rms dw")
    b = _r(1024, seed=15)
    x2, w2 = _r(77, 1024, seed=16), _r(1024, seed=17)
    _close(ops.layer_norm(x2, w2, b, 1e-6), ref.layer_norm(x2, w2, b, 1e-6), name="layernorm")


@pytest.mark.parametrize("D,nq,nkv", [(128, 32, 8), (128, 5, 1), (64, 8, 4), (32, 4, 2)])
def test_qk_norm_rope(D, nq, nkv):
    T = 97
    qkv = _r(T, (nq + 2 * nkv) * D, seed=18)
    qw, kw = (1 + 0.1 * _r(D, seed=19).float()).bfloat16(), (1 + 0.1 * _r(D, seed=20).float()).bfloat16()
    pos = torch.randint(0, 500, (3, T), device=DEV, dtype=torch.int32)
    rope = ops.RopeCfg(D, 5e6, {128: (24, 20, 20), 64: (12, 10, 10)}.get(D, (6, 5, 5)), True)
    q, k, v, rq, rk = ops.qk_norm_rope(qkv, qw, kw, pos, rope, n_q=nq, n_kv=nkv, eps=1e-6)
    qr, kr, vr, rqr, rkr = ref.qk_norm_rope(qkv, qw, kw, pos, n_q=nq, n_kv=nkv, head_dim=D, theta=5e6,
                                            section=rope.section, interleaved=True, eps=1e-6)
    _close(q, qr, name="q")
    _close(k, kr, name="k")
    _close(v, vr, rtol=0, atol=0, name="v")
    dq, dk, dv = _r(T, nq, D, seed=21), _r(T, nkv, D, seed=22), _r(T, nkv, D, seed=23)
    dqw, dkw = torch.zeros(D, device=DEV), torch.zeros(D, device=DEV)
    dqkv = ops.qk_norm_rope_bwd(dq, dk, dv, qkv, qw, kw, pos, rq, rk, rope, n_q=nq, n_kv=nkv, eps=1e-6,
                                dqw_accum=dqw, dkw_accum=dkw)
    dref, dqwr, dkwr = ref.qk_norm_rope_bwd(dq, dk, dv, qkv, qw, kw, pos, rqr, rkr, n_q=nq, n_kv=nkv, head_dim=D,
                                            theta=5e6, section=rope.section, interleaved=True, eps=1e-6)
    _close(dqkv, dref, name="dqkv")
    _close(dqw, dqwr, rtol=1e-3, atol=1e-2, name="dqw")
    _close(dkw, dkwr, rtol=1e-3, atol=1e-2, name="dkw")


@pytest.mark.parametrize("T,norm", [(5111, True), (300, False), (4000, False)])
def test_qk_rope_bwd_large_and_rotation_only(T, norm):
    """Many items per warp (grid-stride weight-gradient accumulation) and the no-q/k-norm variant."""
    D, nq, nkv = 128, 32, 8
    qkv = _r(T, (nq + 2 * nkv) * D, seed=70)
    qw, kw = ((1 + 0.1 * _r(D, seed=71).float()).bfloat16(), (1 + 0.1 * _r(D, seed=72).float()).bfloat16()) \
        if norm else (None, None)
    pos = torch.randint(0, 2000, (3, T), device=DEV, dtype=torch.int32)
    rope = ops.RopeCfg(D, 1e6, (24, 20, 20) if norm else (16, 24, 24), norm)
    q, k, v, rq, rk = ops.qk_norm_rope(qkv, qw, kw, pos, rope, n_q=nq, n_kv=nkv, eps=1e-6)
    qr, kr, vr, rqr, rkr = ref.qk_norm_rope(qkv, qw, kw, pos, n_q=nq, n_kv=nkv, head_dim=D, theta=1e6,
                                            section=rope.section, interleaved=norm, eps=1e-6)
    _close(q, qr, name="q")
    _close(k, kr, name="k")
    dq, dk, dv = _r(T, nq, D, seed=73), _r(T, nkv, D, seed=74), _r(T, nkv, D, seed=75)
    dqw, dkw = torch.zeros(D, device=DEV), torch.zeros(D, device=DEV)
    dqkv = ops.qk_norm_rope_bwd(dq, dk, dv, qkv, qw, kw, pos, rq, rk, rope, n_q=nq, n_kv=nkv, eps=1e-6,
                                dqw_accum=dqw if norm else None, dkw_accum=dkw if norm else None)
    dref, dqwr, dkwr = ref.qk_norm_rope_bwd(dq, dk, dv, qkv, qw, kw, pos, rqr, rkr, n_q=nq, n_kv=nkv, head_dim=D,
                                            theta=1e6, section=rope.section, interleaved=norm, eps=1e-6)
    _close(dqkv, dref, name="dqkv")
    if norm:
        torch.testing.assert_close(dqw, dqwr.float(), rtol=2e-3, atol=2e-1)
        torch.testing.assert_close(dkw, dkwr.float(), rtol=2e-3, atol=2e-1)


@pytest.mark.parametrize("D,Hq,Hkv,causal", [(128, 8, 2, True), (128, 8, 2, False), (64, 4, 4, False), (64, 8, 2, True),
                                             (32, 4, 2, True), (16, 4, 4, False)])
def test_flash_attn(D, Hq, Hkv, causal):
    lens = [1, 63, 64, 130, 388, 17]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    T = sum(lens)
    q, k, v = _r(T, Hq, D, seed=24), _r(T, Hkv, D, seed=25), _r(T, Hkv, D, seed=26)
    scale = 1 / math.sqrt(D)
    o, lse = ops.flash_attn(q, k, v, cu, max(lens), causal=causal, scale=scale)
    orf, lser = ref.flash_attn(q, k, v, cu, max(lens), causal=causal, scale=scale)
    _close(o, orf, name="attn o")
    _close(lse, lser, rtol=1e-3, atol=2e-3, name="attn lse")
    do = _r(T, Hq, D, seed=27)
    dq, dk, dv = ops.flash_attn_bwd(do, q, k, v, o, lse, cu, max(lens), causal=causal, scale=scale)
    dqr, dkr, dvr = ref.flash_attn_bwd(do, q, k, v, orf, lser, cu, max(lens), causal=causal, scale=scale)
    _close(dq, dqr, name="dq")
    _close(dk, dkr, name="dk")
    _close(dv, dvr, name="dv")


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 32, 8), (64, 16, 16)])
def test_flash_attn_shared_prefix(D, Hq, Hkv):
    """Segments that attend to a shared prompt prefix (pack_groups layout): fwd + bwd vs the fp32 oracle."""
    # two groups: prompt lengths 150 / 70, members of lengths (90, 1, 130) / (64, 65)
    layout = [(150, [90, 1, 130]), (70, [64, 65])]
    cu, pre, xq = [0], [], []
    for P, members in layout:
        p0 = cu[-1]
        cu.append(p0 + P)
        pre.append((0, 0))
        slot = len(pre) - 1
        first = cu[-1]
        for n in members:
            cu.append(cu[-1] + n)
            pre.append((p0, P))
            xq.append((0, 0))
        xq.insert(slot, (first, cu[-1]))
    T = cu[-1]
    cu_t = torch.tensor(cu, dtype=torch.int32, device=DEV)
    pre_t = torch.tensor(pre, dtype=torch.int32, device=DEV)
    xq_t = torch.tensor(xq, dtype=torch.int32, device=DEV)
    L = max(b - a for a, b in zip(cu, cu[1:]))
    q, k, v = _r(T, Hq, D, seed=50), _r(T, Hkv, D, seed=51), _r(T, Hkv, D, seed=52)
    scale = 1 / math.sqrt(D)
    o, lse = ops.flash_attn(q, k, v, cu_t, L, causal=True, scale=scale, pre=pre_t)
    orf, lser = ref.flash_attn(q, k, v, cu_t, L, causal=True, scale=scale, pre=pre_t)
    _close(o, orf, name="o")
    torch.testing.assert_close(lse, lser, atol=2e-3, rtol=2e-3)
    do = _r(T, Hq, D, seed=53)
    dq, dk, dv = ops.flash_attn_bwd(do, q, k, v, o, lse, cu_t, L, causal=True, scale=scale, pre=pre_t, xq=xq_t)
    dqr, dkr, dvr = ref.flash_attn_bwd(do, q, k, v, orf, lser, cu_t, L, causal=True, scale=scale, pre=pre_t)
    _close(dq, dqr, name="dq")
    _close(dk, dkr, name="dk")
    _close(dv, dvr, name="dv")


def test_flash_attn_unsupported_head_dim_pads():
    """head_dim 80 (Qwen2.5 ViT) runs on the 128 kernel with zero padding."""
    lens = [196, 64, 300]
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=DEV)
    T = int(cu[-1])
    q, k, v = _r(T, 16, 80, seed=60), _r(T, 16, 80, seed=61), _r(T, 16, 80, seed=62)
    o, lse = ops.flash_attn(q, k, v, cu, max(lens), causal=False)
    orf, lser = ref.flash_attn(q, k, v, cu, max(lens), causal=False, scale=1 / math.sqrt(80))
    _close(o, orf, name="o80")
    torch.testing.assert_close(lse, lser, atol=2e-3, rtol=2e-3)


def test_decode_attn_and_kv_write():
    B, Hq, Hkv, D, Tmax = 5, 32, 8, 128, 300
    kc = torch.zeros(B, Hkv, Tmax, D, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    lens = torch.tensor([1, 17, 128, 299, 200], device=DEV, dtype=torch.int32)
    k, v = _r(int(lens.sum()), Hkv, D, seed=28), _r(int(lens.sum()), Hkv, D, seed=29)
    seq = torch.repeat_interleave(torch.arange(B, device=DEV), lens.long())
    pos = torch.cat([torch.arange(int(n), device=DEV) for n in lens])
    ops.kv_write(k, v, kc, vc, seq, pos)
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    kc2[seq, :, pos] = k
    vc2[seq, :, pos] = v
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    q = _r(B, Hq, D, seed=30)
    _close(ops.decode_attn(q, kc, vc, lens), ref.decode_attn(q, kc, vc, lens, scale=1 / math.sqrt(D)), name="decode")


@pytest.mark.parametrize("B,Hq,Hkv,Tmax", [(3, 32, 8, 1000), (2, 16, 8, 700), (4, 64, 8, 260), (64, 32, 8, 390)])
def test_decode_attn_poisoned_cache(B, Hq, Hkv, Tmax):
    """Cache slots past each length hold NaN: the kernel must not read them into the output."""
    D = 128
    g = torch.Generator(device="cpu").manual_seed(B * 1000 + Tmax)
    lens = torch.randint(1, Tmax + 1, (B,), generator=g).to(DEV, torch.int32)
    lens[0] = Tmax
    kc = _r(B, Hkv, Tmax, D, seed=40)
    vc = _r(B, Hkv, Tmax, D, seed=41)
    pos = torch.arange(Tmax, device=DEV)[None, None, :, None]
    valid = pos < lens.long()[:, None, None, None]
    kp = torch.where(valid, kc, torch.full_like(kc, float("nan")))
    vp = torch.where(valid, vc, torch.full_like(vc, float("nan")))
    q = _r(B, Hq, D, seed=42)
    out = ops.decode_attn(q, kp, vp, lens)
    assert torch.isfinite(out.float()).all()
    _close(out, ref.decode_attn(q, kc * valid, vc * valid, lens, scale=1 / math.sqrt(D)), name="decode_poisoned")


def test_embedding_ops():
    V, H, T = 1000, 256, 77
    table = _r(V, H, seed=31)
    tok = torch.randint(0, V, (T,), device=DEV)
    h = ops.embed(tok, table)
    assert torch.equal(h, table[tok])
    rows = torch.tensor([3, 9, 40], device=DEV)
    src = _r(3, H, seed=32)
    h2 = h.clone()
    ops.scatter_rows_(h2, rows, src, add=True)
    _close(h2, ref.scatter_rows(h, rows, src, True), name="scatter add")
    ops.scatter_rows_(h2, rows, src, add=False)
    assert torch.equal(h2[rows], src)
    dh = _r(T, H, seed=33)
    tok2 = tok.clone()
    tok2[5] = -1
    dt = torch.zeros(V, H, device=DEV)
    ops.embed_bwd(tok2, dh, dt)
    _close(dt, ref.embed_bwd(tok2, dh, torch.zeros(V, H, device=DEV)), rtol=1e-5, atol=1e-5, name="embed bwd")


def test_swiglu_bwd_and_vision_rope():
    pre, da = _r(50, 2 * 384, seed=34), _r(50, 384, seed=35)
    _close(ops.swiglu_bwd(da, pre), ref.swiglu_bwd(da, pre), name="swiglu bwd")
    N, H, D = 64, 16, 64
    qkv = _r(N, 3 * H * D, seed=36)
    rc = torch.randint(0, 40, (N, 2), device=DEV, dtype=torch.int32)
    for style in (0, 1):
        for a, b in zip(ops.vision_rope(qkv, rc, n_heads=H, head_dim=D, style=style),
                        ref.vision_rope(qkv, rc, n_heads=H, head_dim=D, style=style)):
            _close(a, b, name=f"vision rope style {style}")


def test_patchify():
    from vlmrl.utils.vlm import CLIP_MEAN, CLIP_STD

    img = torch.randint(0, 256, (3, 64, 96, 3), device=DEV, dtype=torch.uint8)
    out = ops.patchify_uint8(img, patch=16, temporal=2, merge=2, mean=CLIP_MEAN.tolist(), std=CLIP_STD.tolist())
    exp = ref.patchify_uint8(img, patch=16, temporal=2, merge=2, mean=CLIP_MEAN.tolist(), std=CLIP_STD.tolist())
    _close(out, exp, rtol=1e-2, atol=1e-2, name="patchify")


@pytest.mark.parametrize("M,V,H", [(200, 1000, 128), (1100, 151936, 2560)])
def test_vocab_logprob(M, V, H):
    h, w = _r(M, H, seed=37), _r(V, H, scale=0.05, seed=38)
    tgt = torch.randint(0, V, (M,), device=DEV)
    logp, ent, lse = ops.vocab_logprob(h, w, tgt)
    lr, er, sr = ref.vocab_logprob(h, w, tgt)
    _close(lse, sr, rtol=1e-4, atol=1e-3, name="lse")
    _close(logp, lr, rtol=1e-4, atol=1e-3, name="logp")
    _close(ent, er, rtol=1e-4, atol=1e-3, name="entropy")
    if V > 10000:
        return
    g1, g2 = torch.randn(M, device=DEV), torch.randn(M, device=DEV)
    dw = torch.zeros(V, H, device=DEV)
    dh = ops.vocab_logprob_bwd(h, w, tgt, lse, ent, g1, g2, dw)
    dhr, dwr = ref.vocab_logprob_bwd(h, w, tgt, sr, er, g1, g2)
    _close(dh, dhr, rtol=3e-2, atol=3e-2, name="dh")
    _close(dw, dwr, rtol=3e-2, atol=3e-2, name="dw")
    _no_device_error()


@pytest.mark.parametrize("k,p,temp", [(5, 0.9, 0.7), (50, 0.95, 1.0), (1024, 1.0, 0.7)])
def test_sampler_matches_oracle(k, p, temp):
    B, V = 16, 151936
    logits = torch.randn(B, V, device=DEV) * 3
    tok, lp = ops.sample(logits, temperature=temp, top_k=k, top_p=p, seed=1234, step=7)
    tr, lr = ref.sample(logits.cpu(), temperature=temp, top_k=k, top_p=p, seed=1234, step=7)
    agree = (tok.cpu() == tr).float().mean().item()
    assert agree >= 0.9, f"token agreement {agree}"
    same = tok.cpu() == tr
    torch.testing.assert_close(lp.cpu()[same], lr[same], atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("V,k,p,temp", [(151936, 5, 0.9, 0.7), (151936, 16, 1.0, 1.3), (1000, 1, 0.5, 0.7),
                                        (1000, 7, 0.95, 2.0)])
def test_lm_head_sample_matches_unfused(V, k, p, temp):
    """The lm_head fused with the sampler draws the same tokens with the same log-probs as lm_logits + sample:
    the GEMM tiling is the unfused one, so the logits are bitwise equal, and the merge follows the sampler's
    arithmetic; no [B, V] logits buffer is written (V = 1000 has a partial last tile)."""
    B, H = 64, 2560
    h = _r(B, H, seed=3)
    w = _r(V, H, scale=0.05, seed=4)
    seed = torch.tensor([987654321], dtype=torch.int64, device=DEV)
    for step in (3, 4):
        st = torch.tensor([step], dtype=torch.int64, device=DEV)
        logits = ops.lm_logits(h, w)
        tu, lu = ops.sample(logits, temperature=temp, top_k=k, top_p=p, seed=seed, step=st, row_offset=17)
        tf, lf = ops.lm_head_sample(h, w, temperature=temp, top_k=k, top_p=p, seed=seed, step=st, row_offset=17)
        torch.cuda.synchronize()
        assert torch.equal(tf, tu), (tf != tu).nonzero()
        # V = 151936 uses the same GEMM tiling in both paths (bitwise equal logits); the small vocabulary's
        # unfused lm_head runs stream-K, whose partial-sum order differs in the last bits
        tol = 1e-6 if V == 151936 else 1e-4
        torch.testing.assert_close(lf, lu, atol=tol, rtol=tol)
    _no_device_error()


def test_adamw_and_sqnorm():
    n = 10000
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    p2, g2, m2, v2 = p.cpu().clone(), g.cpu(), m.cpu().clone(), v.cpu().clone()
    ph = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    for step in (1, 2, 3):
        ops.adamw_(p, g, m, v, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=step,
                   grad_scale=0.5, p_half=ph)
        ref.adamw_(p2, g2, m2, v2, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=step,
                   grad_scale=0.5)
    torch.testing.assert_close(p.cpu(), p2, atol=1e-6, rtol=1e-5)
    s = ops.sq_norm(g)
    torch.testing.assert_close(s.cpu()[0], (g2 ** 2).sum(), rtol=1e-4, atol=1e-3)
    for n in (10001, 5_000_016, 7):  # scalar tail path, vectorised grid-stride path, tiny
        x = torch.randn(n, device=DEV)
        torch.testing.assert_close(ops.sq_norm(x).cpu()[0], (x.double() ** 2).sum().float().cpu(), rtol=1e-4, atol=1e-3)


def test_down_dgrad_with_fused_swiglu_backward():
    """The SwiGLU-backward GEMM epilogue equals dgrad followed by the elementwise backward."""
    M, H, F = 777, 512, 1536
    dy, w = _r(M, H, seed=80), _r(H, F, scale=0.05, seed=81)
    pre = _r(M, 2 * F, seed=82)
    fused = ops.grad_input_swiglu(dy, w, pre)
    unfused = ops.swiglu_bwd(ops.grad_input(dy, w), pre)
    torch.testing.assert_close(fused.float(), unfused.float(), atol=1e-2, rtol=1e-2)
    exp = ref.swiglu_bwd(ref.gemm(dy, w, b_kmajor=False, out_dtype=torch.float32).bfloat16(), pre)
    _close(fused, exp, name="dpre")


def test_adamw_vectorised_matches_oracle():
    n = 1000 * 128
    p, g = _r(n, seed=83).float(), _r(n, seed=84).float()
    m, v = _r(n, seed=85).float() * 0.1, _r(n, seed=86).float().abs() * 0.01
    ph = torch.empty(n, dtype=torch.bfloat16, device=DEV)
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    ops.adamw_(p, g, m, v, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=3, grad_scale=0.5,
               p_half=ph)
    ref.adamw_(pr, g, mr, vr, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=3, grad_scale=0.5)
    torch.testing.assert_close(p, pr, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(m, mr, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(v, vr, atol=1e-7, rtol=1e-5)
    assert torch.equal(ph, p.bfloat16())


@pytest.mark.parametrize("M,H", [(5111, 2560), (37, 4096), (1, 128)])
def test_rms_norm_bwd_weight_grad_and_residual_add(M, H):
    x, dy, w = _r(M, H, seed=90), _r(M, H, seed=91), (1 + 0.1 * _r(H, seed=92).float()).bfloat16()
    add = _r(M, H, seed=93)
    y, rstd = ops.rms_norm(x, w, 1e-6)
    dw = torch.zeros(H, device=DEV)
    dx = ops.rms_norm_bwd(dy, x, w, rstd, dw_accum=dw, add=add)
    dxr, dwr = ref.rms_norm_bwd(dy, x, w, rstd)
    _close(dx, (dxr.float() + add.float()), name="dx+add")
    torch.testing.assert_close(dw, dwr.float(), rtol=2e-3, atol=5e-2)


def test_bounded_peer_wait_reports_timeout_and_context_survives():
    """A flag that nothing ever sets: the wait gives up after its (short) budget, the host gets a
    CollectiveTimeout, and the GPU keeps working."""
    from vlmrl.ops import CollectiveTimeout
    from vlmrl.ops._ext import ext

    sig = torch.zeros(4, dtype=torch.int64, device=DEV)          # slot 0, world 2: peer 1's counter stays 0
    ext().peer_wait(sig.data_ptr(), 0, 1, 0, 2, torch.cuda.current_device(), 2_000_000)   # ~1 ms budget
    with pytest.raises(CollectiveTimeout):
        ops.check_errors()
    x = _r(256, 256, seed=99)
    _close(ops.gemm(x, x), ref.gemm(x, x, out_dtype=torch.float32), name="after timeout")
    _no_device_error()


def _sharded_unit(W, rows, cols, lead, seed=0):
    """A flat bf16 unit [lead elements | rows x cols matrix | tail] split into W separately allocated shards
    (W emulated ranks on one GPU); returns (full unit, shard tensors, shard bytes, matrix offset)."""
    numel = lead + rows * cols + 128
    P = -(-numel // (128 * W)) * 128 * W
    full = _r(P, seed=seed)
    n = P // W
    shards = [full[r * n:(r + 1) * n].clone() for r in range(W)]
    return full, shards, n * 2, lead


@pytest.mark.parametrize("W", [1, 3, 8])
@pytest.mark.parametrize("M", [64, 700, 2100, 6000])
def test_gemm_with_fused_weight_gather(W, M):
    """GEMMs whose weight operand is assembled from W shards inside the kernel match the plain GEMM on the
    full matrix, for the forward (K-major), dgrad (MN-major) and SwiGLU epilogue, and re-launch cleanly.
    M covers 128- and 256-wide tiles and CTAs that own one or several tiles."""
    N, K = 1344, 576
    full, shards, SB, lead = _sharded_unit(W, N, K, 256)
    w_full = full[lead:lead + N * K].view(N, K)
    dst = torch.full_like(full, 7.0)
    flags = torch.zeros(4096, dtype=torch.int32, device=DEV)
    ctr = torch.zeros(2, dtype=torch.int32, device=DEV)
    srcs = [s.data_ptr() for s in shards]
    sw = ops.ShardedWeight(dst[lead:lead + N * K].view(N, K), srcs, dst.data_ptr(), SB, flags, ctr)
    x = _r(M, K, seed=1)
    for rep in range(2):
        dst.fill_(7.0)
        y = ops.linear(x, sw)
        _close(y, x.float() @ w_full.float().T, name=f"fwd rep {rep}")
        assert torch.equal(dst[lead:lead + N * K], full[lead:lead + N * K])
    dst.fill_(-3.0)
    dy = _r(M, N, seed=2)
    dx = ops.grad_input(dy, sw)
    _close(dx, dy.float() @ w_full.float(), name="dgrad")
    dst.fill_(7.0)
    act, pre = ops.linear_swiglu(x, sw)
    pre_ref = x.float() @ w_full.float().T
    _close(pre, pre_ref, name="swiglu pre")
    _close(act, ref.swiglu_interleaved(pre_ref.bfloat16().float()), name="swiglu act")
    torch.cuda.synchronize()
    assert int(flags.abs().sum()) == 0 and int(ctr.abs().sum()) == 0  # the last CTA reset the counters
    _no_device_error()


def test_unit_gather_ranges():
    W = 4
    full, shards, SB, lead = _sharded_unit(W, 96, 64, 256, seed=3)
    dst = torch.zeros_like(full)
    ranges = [(0, lead * 2), ((lead + 96 * 64) * 2, full.numel() * 2)]
    ops.unit_gather([s.data_ptr() for s in shards], dst.data_ptr(), SB, ranges)
    for a, b in ranges:
        assert torch.equal(dst[a // 2:b // 2], full[a // 2:b // 2])
    assert int(dst[lead:lead + 96 * 64].abs().sum()) == 0
    _no_device_error()


@pytest.mark.parametrize("B", [3, 64])
@pytest.mark.parametrize("norm", [True, False])
def test_decode_gemms_with_fused_consumers_match_separate_kernels(B, norm):
    """The decode GEMMs that run their consumer after a grid-wide barrier (one launch) produce what the
    stream-K GEMM followed by the separate consumer kernel produces, and replay from a CUDA graph."""
    nq, nkv, D, H, F, Tmax = 8, 2, 128, 1024, 2048, 96
    rope = ops.RopeCfg(D, 5e6, (24, 20, 20), True)
    x = _r(B, H, seed=1)
    w_qkv = _r((nq + 2 * nkv) * D, H, scale=0.03, seed=2)
    bias = _r((nq + 2 * nkv) * D, scale=0.1, seed=3)
    qw, kw = (_r(D, seed=4) + 1, _r(D, seed=5) + 1) if norm else (None, None)
    g = torch.Generator(device=DEV).manual_seed(6)
    lens = torch.randint(0, Tmax - 1, (B,), generator=g, device=DEV, dtype=torch.int32)
    delta = torch.randint(-5, 5, (B,), generator=g, device=DEV, dtype=torch.int64)
    caches = [(torch.zeros(B, nkv, Tmax, D, dtype=torch.bfloat16, device=DEV),
               torch.zeros(B, nkv, Tmax, D, dtype=torch.bfloat16, device=DEV)) for _ in range(2)]
    ws, meta = ops.gemm_partials(x, w_qkv)
    q1 = ops.dec_qkv(ws, meta, bias, qw, kw, lens, delta, rope, *caches[0], n_q=nq, n_kv=nkv, eps=1e-6)
    q2 = ops.dec_linear_qkv(x, w_qkv, bias, qw, kw, lens, delta, rope, *caches[1], n_q=nq, n_kv=nkv, eps=1e-6)
    _close(q2, q1, rtol=1e-2, atol=1e-2, name="q")
    _close(caches[1][0], caches[0][0], rtol=1e-2, atol=1e-2, name="k cache")
    _close(caches[1][1], caches[0][1], rtol=1e-2, atol=1e-2, name="v cache")

    res = _r(B, H, seed=7)
    w_o, nw = _r(H, nq * D, scale=0.03, seed=8), _r(H, seed=9) + 1
    o = _r(B, nq * D, seed=10)
    ws, meta = ops.gemm_partials(o, w_o)
    h1, hn1 = ops.dec_residual_norm(ws, meta, res, nw, 1e-6)
    h2, hn2 = ops.dec_linear_residual_norm(o, w_o, res, nw, 1e-6)
    _close(h2, h1, rtol=1e-2, atol=1e-2, name="h")
    _close(hn2, hn1, rtol=1e-2, atol=1e-2, name="hn")

    w_gu = _r(2 * F, H, scale=0.03, seed=11)
    ws, meta = ops.gemm_partials(hn1, w_gu)
    a1 = ops.dec_swiglu(ws, meta)
    a2 = ops.dec_linear_swiglu(hn1, w_gu)
    _close(a2, a1, rtol=1e-2, atol=1e-2, name="swiglu")

    # graph replay: the grid barrier resets itself between launches
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        a3 = ops.dec_linear_swiglu(hn1, w_gu)
        h3, hn3 = ops.dec_linear_residual_norm(o, w_o, res, nw, 1e-6)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    _close(a3, a1, rtol=1e-2, atol=1e-2, name="swiglu (graph)")
    _close(hn3, hn1, rtol=1e-2, atol=1e-2, name="hn (graph)")
    _no_device_error()


def test_decode_attn_reads_shared_prompt_from_group_leader(monkeypatch):
    """With lead/share_len, whole key chunks inside a row's shared prompt come from the leader's row: the
    members' own copies of the prompt are never read (here they are NaN) and the result equals the
    attention over clean copies.  One key split, so chunks start at multiples of 64."""
    monkeypatch.setenv("VLMRL_DECODE_SPLITS", "1")
    B, gs, Hq, Hkv, D, Tmax = 8, 4, 8, 2, 128, 320
    g = torch.Generator(device=DEV).manual_seed(3)
    kc = _r(B, Hkv, Tmax, D, seed=4)
    vc = _r(B, Hkv, Tmax, D, seed=5)
    plen = torch.tensor([200, 200, 200, 200, 137, 137, 137, 137], dtype=torch.int32, device=DEV)
    for b in range(B):
        lead = b // gs * gs
        kc[b, :, :int(plen[b])] = kc[lead, :, :int(plen[b])]
        vc[b, :, :int(plen[b])] = vc[lead, :, :int(plen[b])]
    lens = plen + torch.randint(1, 100, (B,), generator=g, device=DEV, dtype=torch.int32)
    q = _r(B, Hq, D, seed=6)
    ref_o = ops.decode_attn(q, kc, vc, lens)
    lead = (torch.arange(B, device=DEV, dtype=torch.int32) // gs) * gs
    kp, vp = kc.clone(), vc.clone()
    for b in range(B):
        if b % gs:  # poison the members' whole-chunk prompt copies
            n = int(plen[b]) // 64 * 64
            kp[b, :, :n] = float("nan")
            vp[b, :, :n] = float("nan")
    out = ops.decode_attn(q, kp, vp, lens, lead=lead, share_len=plen)
    assert torch.isfinite(out.float()).all()
    _close(out, ref_o, rtol=1e-2, atol=1e-2, name="shared-prompt decode attention")
    _no_device_error()


@pytest.mark.parametrize("M,N,K", [(520, 272, 200), (2304, 1536, 640), (4608, 2304, 256)])
def test_gemm_cta_pair_tiles(M, N, K):
    """GEMMs with M >= 512 run as CTA pairs (256 x 256 tiles, tcgen05 cta_group::2, half of B per CTA). Ragged
    M / N, every operand layout and every epilogue against the fp32 oracle, twice in a row."""
    a, w = _r(M, K, seed=70), _r(N, K, scale=0.1, seed=71)
    bias, res = _r(N, seed=72), _r(M, N, seed=73)
    for rep in range(2):
        _close(ops.gemm(a, w, bias=bias, residual=res), ref.gemm(a, w, bias=bias, residual=res, out_dtype=torch.float32),
               name=f"pair nt+epi rep {rep}")
    _close(ops.gemm(a, w, out_dtype=torch.float32), ref.gemm(a, w, out_dtype=torch.float32), rtol=5e-3, atol=5e-3,
           name="pair nt f32")
    act, pre = ops.linear_swiglu(a, w)
    pre_ref = ref.gemm(a, w, out_dtype=torch.float32)
    _close(pre, pre_ref, name="pair swiglu pre")
    _close(act, ref.swiglu_interleaved(pre_ref.to(torch.bfloat16)), name="pair swiglu")
    out = ops.gemm(a, w, bias=bias, epilogue=ops.EPI_GELU_TANH)
    _close(out, ref.gelu(ref.gemm(a, w, bias=bias, out_dtype=torch.float32), "tanh"), name="pair gelu")
    dy = _r(M, N, seed=74)
    _close(ops.grad_input(dy, w), dy.float() @ w.float(), name="pair dgrad")
    x = _r(M, K, seed=75)
    acc = torch.ones(N, K, device=DEV)
    ops.grad_weight(dy, x, accumulate=acc)
    _close(acc, dy.float().t() @ x.float() + 1.0, rtol=5e-3, atol=5e-3, name="pair wgrad acc")
    _no_device_error()


@pytest.mark.parametrize("M,N,K", [(1, 2560, 4096), (8, 6144, 2560), (17, 1000, 2560), (64, 2560, 9728), (64, 6144, 2560)])
def test_decode_partials(M, N, K):
    """The decode-shaped partial-sum GEMM (stream-K layout; the skinny mma.sync kernel when it is selected)
    summed by the residual + RMSNorm consumer equals x @ w.T; ragged M and N, inside and outside the
    static-weights mode."""
    x, w = _r(M, K, seed=80), _r(N, K, scale=0.02, seed=81)
    zero = torch.zeros(M, N, dtype=torch.bfloat16, device=DEV)
    ones = torch.ones(N, dtype=torch.bfloat16, device=DEV)
    want = x.float() @ w.float().T
    for static in (False, True):
        with ops.static_weights() if static else torch.no_grad():
            ws, meta = ops.gemm_partials(x, w)
            h, _ = ops.dec_residual_norm(ws, meta, zero, ones, 1e-6)
        _close(h, want, name=f"skinny partials static={static}")
    _no_device_error()


def test_tcgen05_dkdv_backward_matches_oracle():
    """The tcgen05 dK / dV backward (opt-in, VLMRL_ATTN_BWD_TC=1; the switch is read once per process, so
    the comparison runs in a child process): causal GQA and shared-prefix segments against the fp32 oracle."""
    import os
    import subprocess
    import sys

    code = r"""
import math, torch
from vlmrl import ops
from vlmrl.ops import reference as ref
def r(*s, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*s, generator=g, device="cuda").bfloat16()
for D, Hq, Hkv in ((128, 8, 2), (64, 4, 4)):
    lens = [1, 63, 130, 388, 17]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
    T = sum(lens)
    q, k, v, do = r(T, Hq, D, seed=1), r(T, Hkv, D, seed=2), r(T, Hkv, D, seed=3), r(T, Hq, D, seed=4)
    sc = 1 / math.sqrt(D)
    o, lse = ops.flash_attn(q, k, v, cu, max(lens), causal=True, scale=sc)
    dq, dk, dv = ops.flash_attn_bwd(do, q, k, v, o, lse, cu, max(lens), causal=True, scale=sc)
    orf, lr = ref.flash_attn(q, k, v, cu, max(lens), causal=True, scale=sc)
    _, dkr, dvr = ref.flash_attn_bwd(do, q, k, v, orf, lr, cu, max(lens), causal=True, scale=sc)
    for a, b, n in ((dk, dkr, "dk"), (dv, dvr, "dv")):
        err = (a.float() - b.float()).abs().max().item()
        lim = 2e-2 + 2e-2 * b.float().abs().max().item()
        assert err <= lim, (D, n, err, lim)
from vlmrl.ops._ext import ext
assert ext().read_and_clear_error(torch.cuda.current_device()) == 0
print("ok")
"""
    env = dict(os.environ, VLMRL_ATTN_BWD_TC="1")
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stdout[-2000:] + res.stderr[-2000:]
