"""PyTorch reference implementations of every hot op (the test oracle and the CPU path).

Each function here is the contract of a CUDA kernel in ``csrc/``: same
arguments, same layouts, fp32 math.  Layout conventions shared by all ops:

* activations are packed token-major ``[T, features]`` (no padding; sequences
  delimited by ``cu_seqlens`` int32 ``[B+1]``);
* weights use the PyTorch ``[out, in]`` layout, so ``linear`` is ``x @ w.T``;
* the fused gate/up weight interleaves rows: row ``2j`` is gate_j, row
  ``2j+1`` is up_j, so one GEMM tile holds matching gate/up columns;
* attention tensors are ``[T, heads, head_dim]``; ``lse`` is ``[heads, T]``.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from vlmrl.models.qwen3vl.rope import mrope_axis_map, inv_freq


def _f(x: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if x is None else x.float()


# ------------------------------------------------------------------ GEMM family
def gemm(a: torch.Tensor, b: torch.Tensor, *, a_kmajor: bool = True, b_kmajor: bool = True,
         bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
         alpha: float = 1.0, out_dtype: torch.dtype = torch.bfloat16,
         accumulate: Optional[torch.Tensor] = None) -> torch.Tensor:
    """D[M,N] = alpha * A·Bᵀ (+ bias[N]) (+ residual[M,N]) (+ accumulate[M,N]).

    ``a_kmajor``: A stored [M,K] (else stored [K,M]); ``b_kmajor``: B stored
    [N,K] (else stored [K,N]).
    """
    A = a.float() if a_kmajor else a.float().t()
    B = b.float() if b_kmajor else b.float().t()
    d = alpha * (A @ B.t())
    if bias is not None:
        d = d + bias.float()
    if residual is not None:
        d = d + residual.float()
    if accumulate is not None:
        d = d + accumulate.float()
        accumulate.copy_(d.to(accumulate.dtype))
        return accumulate
    return d.to(out_dtype)


def linear(x, w, bias=None, residual=None, out_dtype=torch.bfloat16):
    return gemm(x, w, bias=bias, residual=residual, out_dtype=out_dtype)


def swiglu_interleaved(pre: torch.Tensor) -> torch.Tensor:
    """pre [M, 2F] interleaved (gate, up) -> silu(gate) * up [M, F]."""
    p = pre.float()
    g, u = p[:, 0::2], p[:, 1::2]
    return F.silu(g) * u


def linear_swiglu(x, w_gu, out_dtype=torch.bfloat16):
    pre = gemm(x, w_gu, out_dtype=torch.float32)
    return swiglu_interleaved(pre).to(out_dtype), pre.to(out_dtype)


def swiglu_bwd(d_act: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    p = pre.float()
    g, u = p[:, 0::2], p[:, 1::2]
    s = torch.sigmoid(g)
    silu = g * s
    da = d_act.float()
    dg = da * u * (s * (1.0 + g * (1.0 - s)))
    du = da * silu
    out = torch.empty_like(p)
    out[:, 0::2] = dg
    out[:, 1::2] = du
    return out.to(pre.dtype)


def gelu(x: torch.Tensor, approximate: str = "tanh") -> torch.Tensor:
    return F.gelu(x.float(), approximate=approximate)


# ------------------------------------------------------------------ norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = (xf * rstd).to(x.dtype).float() * w.float()   # HF: normalise, cast to input dtype, then scale
    return y.to(x.dtype), rstd.squeeze(-1)


def rms_norm_bwd(dy, x, w, rstd) -> Tuple[torch.Tensor, torch.Tensor]:
    xf, dyf, wf = x.float(), dy.float(), w.float()
    r = rstd.float().unsqueeze(-1)
    xhat = xf * r
    g = dyf * wf
    dx = r * (g - xhat * (g * xhat).mean(-1, keepdim=True))
    dw = (dyf * xhat).reshape(-1, x.shape[-1]).sum(0)
    return dx.to(x.dtype), dw


def layer_norm(x, w, b, eps: float):
    return F.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float() if b is not None else None, eps).to(x.dtype)


# ------------------------------------------------------------------ rotary
def rope_tables(pos: torch.Tensor, head_dim: int, theta: float, section: Sequence[int], interleaved: bool):
    half = head_dim // 2
    axis = torch.from_numpy(mrope_axis_map(section, half, interleaved)).long().to(pos.device)
    freq = torch.from_numpy(inv_freq(head_dim, theta)).to(pos.device)
    ang = pos.float()[axis].t() * freq[None, :]          # [T, half]
    return torch.cos(ang), torch.sin(ang)


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, sign: float = 1.0) -> torch.Tensor:
    """x [T, H, D] fp32 rotated by +/- angle; cos/sin [T, D/2]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sign * sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def qk_norm_rope(qkv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor, pos: torch.Tensor, *,
                 n_q: int, n_kv: int, head_dim: int, theta: float, section: Sequence[int],
                 interleaved: bool, eps: float):
    """qkv [T, (n_q+2n_kv)*D] -> q [T,n_q,D], k [T,n_kv,D], v [T,n_kv,D], rstd_q [T,n_q], rstd_k [T,n_kv].

    Per-head RMSNorm (fp32 statistics, weight [D]) on q and k, then MRoPE on
    both; v is a plain slice.  Output dtype = qkv dtype.
    """
    T = qkv.shape[0]
    D = head_dim
    x = qkv.float().view(T, n_q + 2 * n_kv, D)
    q, k, v = x[:, :n_q], x[:, n_q:n_q + n_kv], x[:, n_q + n_kv:]
    if q_w is None:   # rotation only (attention without q/k RMSNorm)
        rq = torch.ones(q.shape[:2], device=qkv.device)
        rk = torch.ones(k.shape[:2], device=qkv.device)
        qn, kn = q, k
    else:
        rq = torch.rsqrt(q.pow(2).mean(-1) + eps)
        rk = torch.rsqrt(k.pow(2).mean(-1) + eps)
        qn = q * rq[..., None] * q_w.float()
        kn = k * rk[..., None] * k_w.float()
    cos, sin = rope_tables(pos, D, theta, section, interleaved)
    dt = qkv.dtype
    return (_rotate(qn, cos, sin).to(dt), _rotate(kn, cos, sin).to(dt), v.to(dt).contiguous(), rq, rk)


def qk_norm_rope_bwd(dq, dk, dv, qkv, q_w, k_w, pos, rq, rk, *, n_q, n_kv, head_dim, theta, section,
                     interleaved, eps):
    T, D = qkv.shape[0], head_dim
    x = qkv.float().view(T, n_q + 2 * n_kv, D)
    q, k = x[:, :n_q], x[:, n_q:n_q + n_kv]
    cos, sin = rope_tables(pos, D, theta, section, interleaved)
    dqn = _rotate(dq.float(), cos, sin, sign=-1.0)
    dkn = _rotate(dk.float(), cos, sin, sign=-1.0)

    def norm_bwd(g, xin, r, w):
        xhat = xin * r[..., None]
        gw = g * w.float()
        dx = r[..., None] * (gw - xhat * (gw * xhat).mean(-1, keepdim=True))
        return dx, (g * xhat).reshape(-1, D).sum(0)

    if q_w is None:
        dq_in, dqw, dk_in, dkw = dqn, None, dkn, None
    else:
        dq_in, dqw = norm_bwd(dqn, q, rq, q_w)
        dk_in, dkw = norm_bwd(dkn, k, rk, k_w)
    dqkv = torch.cat([dq_in, dk_in, dv.float()], dim=1).reshape(T, -1)
    return dqkv.to(qkv.dtype), dqw, dkw


def vision_rope(qkv: torch.Tensor, rc: torch.Tensor, *, n_heads: int, head_dim: int, theta: float = 10000.0,
                style: int = 0):
    """ViT: qkv [N, 3*H*D] (q|k|v, head-major) -> q, k, v [N, H, D] with 2-D rotary on q, k.

    ``style`` 0: HF (D/4 frequencies per axis, one angle per rotation pair).  ``style`` 1: the reference's
    Qwen3-VL tower (reference ``models/qwen3vl/vision.py:21-30,69-77,226-230,280-284``): D/2 frequencies
    ``theta**(-j/(D/2))``; element j of the first half turns by ``row * f_j`` and element j of the second
    half by ``col * f_j``, through ``x * cos + rotate_half(x) * sin``.
    """
    N, D = qkv.shape[0], head_dim
    x = qkv.float().view(N, 3, n_heads, D)
    rdim = D // 2
    dt = qkv.dtype
    if style == 1:
        freq = 1.0 / (theta ** (torch.arange(0, rdim, dtype=torch.float32, device=qkv.device) / rdim))
        a = rc[:, 0:1].float() * freq[None]  # [N, D/2]
        b = rc[:, 1:2].float() * freq[None]
        cos = torch.cat([torch.cos(a), torch.cos(b)], dim=-1)[:, None, :]
        sin = torch.cat([torch.sin(a), torch.sin(b)], dim=-1)[:, None, :]

        def rot(t):
            t1, t2 = t[..., :rdim], t[..., rdim:]
            return t * cos + torch.cat([-t2, t1], dim=-1) * sin

        return rot(x[:, 0]).to(dt), rot(x[:, 1]).to(dt), x[:, 2].to(dt).contiguous()
    freq = 1.0 / (theta ** (torch.arange(0, rdim, 2, dtype=torch.float32, device=qkv.device) / rdim))
    ang = torch.cat([rc[:, 0:1].float() * freq[None], rc[:, 1:2].float() * freq[None]], dim=-1)  # [N, D/2]
    cos, sin = torch.cos(ang), torch.sin(ang)
    return (_rotate(x[:, 0], cos, sin).to(dt), _rotate(x[:, 1], cos, sin).to(dt), x[:, 2].to(dt).contiguous())


# ------------------------------------------------------------------ attention
def _seg_keys(k, v, s, e, pre, b, rep):
    """Keys/values of segment b ([Hq, P + L, D]) and the prefix length P (shared-prefix segments)."""
    ps, pl = (int(pre[b, 0]), int(pre[b, 1])) if pre is not None else (0, 0)
    kk = torch.cat([k[ps:ps + pl], k[s:e]]).float().transpose(0, 1).repeat_interleave(rep, 0)
    vv = torch.cat([v[ps:ps + pl], v[s:e]]).float().transpose(0, 1).repeat_interleave(rep, 0)
    return kk, vv, ps, pl


def _seg_mask(L: int, pl: int, causal: bool, device):
    mask = torch.zeros(L, pl + L, dtype=torch.bool, device=device)
    if causal:
        mask[:, pl:] = torch.ones(L, L, dtype=torch.bool, device=device).triu(1)
    return mask


def flash_attn(q, k, v, cu_seqlens: torch.Tensor, max_seqlen: int, *, causal: bool, scale: float, pre=None):
    """Varlen GQA attention. Returns (o [T,Hq,D] in q.dtype, lse [Hq,T] fp32).

    ``pre[b] = (start, len)``: the queries of segment b also attend, without a causal mask, to the
    keys of rows [start, start + len) (a prefix shared by several segments).
    """
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    o = torch.empty(T, Hq, D, dtype=torch.float32, device=q.device)
    lse = torch.empty(Hq, T, dtype=torch.float32, device=q.device)
    cu = cu_seqlens.tolist()
    pre = pre.cpu() if pre is not None else None
    for b in range(len(cu) - 1):
        s, e = cu[b], cu[b + 1]
        if e <= s:
            continue
        qb = q[s:e].float().transpose(0, 1)                        # [Hq, L, D]
        kb, vb, _, pl = _seg_keys(k, v, s, e, pre, b, rep)
        sc = (qb @ kb.transpose(1, 2)) * scale
        sc = sc.masked_fill(_seg_mask(e - s, pl, causal, q.device), float("-inf"))
        l = torch.logsumexp(sc, dim=-1)
        p = torch.exp(sc - l[..., None])
        o[s:e] = (p @ vb).transpose(0, 1)
        lse[:, s:e] = l
    return o.to(q.dtype), lse


def flash_attn_bwd(do, q, k, v, o, lse, cu_seqlens, max_seqlen, *, causal: bool, scale: float, pre=None):
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    dq = torch.zeros(T, Hq, D, dtype=torch.float32, device=q.device)
    dk = torch.zeros(T, Hkv, D, dtype=torch.float32, device=q.device)
    dv = torch.zeros(T, Hkv, D, dtype=torch.float32, device=q.device)
    cu = cu_seqlens.tolist()
    pre = pre.cpu() if pre is not None else None
    for b in range(len(cu) - 1):
        s, e = cu[b], cu[b + 1]
        if e <= s:
            continue
        L = e - s
        qb = q[s:e].float().transpose(0, 1)
        kb, vb, ps, pl = _seg_keys(k, v, s, e, pre, b, rep)
        dob = do[s:e].float().transpose(0, 1)
        ob = o[s:e].float().transpose(0, 1)
        sc = (qb @ kb.transpose(1, 2)) * scale
        sc = sc.masked_fill(_seg_mask(L, pl, causal, q.device), float("-inf"))
        p = torch.exp(sc - lse[:, s:e, None])
        dvb = p.transpose(1, 2) @ dob
        dp = dob @ vb.transpose(1, 2)
        delta = (dob * ob).sum(-1, keepdim=True)
        ds = p * (dp - delta) * scale
        dqb = ds @ kb
        dkb = ds.transpose(1, 2) @ qb
        dq[s:e] = dqb.transpose(0, 1)
        dkr = dkb.view(Hkv, rep, pl + L, D).sum(1).transpose(0, 1)
        dvr = dvb.view(Hkv, rep, pl + L, D).sum(1).transpose(0, 1)
        dk[s:e] += dkr[pl:]
        dv[s:e] += dvr[pl:]
        if pl:
            dk[ps:ps + pl] += dkr[:pl]
            dv[ps:ps + pl] += dvr[:pl]
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def decode_attn(q, k_cache, v_cache, lengths, *, scale: float):
    """q [B,Hq,D]; caches [B,Hkv,Tmax,D]; lengths [B] valid entries (incl. the current token)."""
    B, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    rep = Hq // Hkv
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(lengths[b])
        kb = k_cache[b, :, :L].float().repeat_interleave(rep, 0)   # [Hq, L, D]
        vb = v_cache[b, :, :L].float().repeat_interleave(rep, 0)
        sc = (q[b].float()[:, None, :] @ kb.transpose(1, 2)).squeeze(1) * scale   # [Hq, L]
        p = torch.softmax(sc, dim=-1)
        out[b] = (p[:, None, :] @ vb).squeeze(1)
    return out.to(q.dtype)


# ------------------------------------------------------------------ embedding / scatter
def embed(tokens: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    return table[tokens.long()]


def scatter_rows(h: torch.Tensor, rows: torch.Tensor, src: torch.Tensor, add: bool) -> torch.Tensor:
    out = h.clone()
    if add:
        out[rows.long()] = (out[rows.long()].float() + src.float()).to(h.dtype)
    else:
        out[rows.long()] = src.to(h.dtype)
    return out


def embed_bwd(tokens: torch.Tensor, dh: torch.Tensor, dtable: torch.Tensor) -> torch.Tensor:
    """dtable[tokens[t]] += dh[t]; rows with a negative token id are skipped."""
    keep = tokens >= 0
    dtable.index_add_(0, tokens[keep].long(), dh[keep].float())
    return dtable


# ------------------------------------------------------------------ vocab (fused lm_head)
def vocab_logprob(h: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, *, chunk: int = 4096):
    """h [M,H], w [V,H], targets [M] -> (logp[target], entropy, lse), all fp32 [M].

    Logits are computed in fp32 from bf16 operands; only ``chunk`` rows are
    materialised at a time.
    """
    M = h.shape[0]
    logp = torch.empty(M, dtype=torch.float32, device=h.device)
    ent = torch.empty_like(logp)
    lse = torch.empty_like(logp)
    for s in range(0, M, chunk):
        e = min(M, s + chunk)
        z = h[s:e].float() @ w.float().t()
        l = torch.logsumexp(z, dim=-1)
        p = torch.exp(z - l[:, None])
        lse[s:e] = l
        logp[s:e] = z.gather(1, targets[s:e].long()[:, None]).squeeze(1) - l
        ent[s:e] = l - (p * z).sum(-1)
    return logp, ent, lse


def vocab_logprob_bwd(h, w, targets, lse, ent, g_logp, g_ent, *, chunk: int = 4096):
    """Gradients of sum(g_logp*logp + g_ent*entropy) -> (dh [M,H] fp32, dw [V,H] fp32).

    dlogits = g_logp*(onehot - p) - g_ent * p * (log p + H).
    """
    M = h.shape[0]
    dh = torch.empty(M, h.shape[1], dtype=torch.float32, device=h.device)
    dw = torch.zeros(w.shape, dtype=torch.float32, device=h.device)
    for s in range(0, M, chunk):
        e = min(M, s + chunk)
        z = h[s:e].float() @ w.float().t()
        logp_all = z - lse[s:e, None]
        p = torch.exp(logp_all)
        dz = -g_logp[s:e, None] * p - g_ent[s:e, None] * p * (logp_all + ent[s:e, None])
        dz.scatter_add_(1, targets[s:e].long()[:, None], g_logp[s:e, None].float())
        dh[s:e] = dz @ w.float()
        dw += dz.t() @ h[s:e].float()
    return dh, dw


def lm_logits(h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return h.float() @ w.float().t()


# ------------------------------------------------------------------ sampling
def philox_uniform(seed: int, row: torch.Tensor, step: int) -> torch.Tensor:
    """Counter-based uniform in (0,1) per row — must match the CUDA sampler bit-for-bit."""
    from vlmrl.ops.philox import philox_uniform_np

    import numpy as np

    u = philox_uniform_np(int(seed), row.cpu().numpy().astype(np.uint64), int(step))
    return torch.from_numpy(u).to(row.device)


def sample(logits: torch.Tensor, *, temperature: float, top_k: int, top_p: float, seed: int, step: int,
           row_offset: int = 0):
    """Temperature -> top-k shortlist -> nucleus -> inverse-CDF draw with a Philox uniform.

    Returns (token [B] int64, logprob [B] fp32 of the token under the masked,
    tempered distribution — the reference sampler's convention).
    """
    B, V = logits.shape
    z = logits.float() / float(temperature)
    k = V if (top_k is None or top_k <= 0) else min(int(top_k), V)
    vals, idx = torch.topk(z, k, dim=-1)            # sorted descending; ties -> lower index first
    probs = torch.softmax(vals, dim=-1)
    if top_p is not None and 0.0 < float(top_p) < 1.0:
        cum = torch.cumsum(probs, dim=-1)
        keep = cum <= float(top_p)
        keep[:, 0] = True
        vals = torch.where(keep, vals, torch.full_like(vals, float("-inf")))
        probs = torch.softmax(vals, dim=-1)
    u = philox_uniform(seed, torch.arange(B, device=logits.device) + row_offset, step)
    cdf = torch.cumsum(probs, dim=-1)
    choice = torch.searchsorted(cdf, u[:, None].to(cdf.dtype)).squeeze(1).clamp(max=k - 1)
    # never select a masked entry
    nkeep = torch.isfinite(vals).sum(-1)
    choice = torch.minimum(choice, nkeep - 1)
    tok = idx.gather(1, choice[:, None]).squeeze(1)
    lp = torch.log(probs.gather(1, choice[:, None]).squeeze(1))
    return tok, lp


# ------------------------------------------------------------------ optimizer
def adamw_(p: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor, *, lr: float, beta1: float,
           beta2: float, eps: float, weight_decay: float, step: int, grad_scale: float = 1.0,
           p_half: Optional[torch.Tensor] = None) -> None:
    """optax.adamw semantics (bias-corrected moments; decoupled decay added to the update, times lr)."""
    gf = g.float() * grad_scale
    m.mul_(beta1).add_(gf, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(gf, gf, value=1 - beta2)
    mhat = m / (1 - beta1 ** step)
    vhat = v / (1 - beta2 ** step)
    upd = mhat / (vhat.sqrt() + eps) + weight_decay * p
    p.add_(upd, alpha=-lr)
    if p_half is not None:
        p_half.copy_(p.to(p_half.dtype))


def sq_norm(x: torch.Tensor) -> torch.Tensor:
    return x.float().pow(2).sum()


# ------------------------------------------------------------------ vision input
def patchify_uint8(images: torch.Tensor, *, patch: int, temporal: int, merge: int, mean, std) -> torch.Tensor:
    """images [N, H, W, 3] uint8 -> rows [N*gh*gw, 3*temporal*patch*patch] (single frame repeated)."""
    N, H, W, C = images.shape
    x = images.float() / 255.0
    x = (x - torch.tensor(mean, device=x.device)) / torch.tensor(std, device=x.device)
    x = x.permute(0, 3, 1, 2)                      # N, C, H, W
    gh, gw = H // patch, W // patch
    x = x.reshape(N, C, gh // merge, merge, patch, gw // merge, merge, patch)
    x = x.permute(0, 2, 5, 3, 6, 1, 4, 7)          # N, hb, wb, hm, wm, C, py, px
    x = x.unsqueeze(6).expand(N, gh // merge, gw // merge, merge, merge, C, temporal, patch, patch)
    return x.reshape(N * gh * gw, C * temporal * patch * patch)


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "math", "torch", "F")]
