"""Hot ops: hand-written sm_100a CUDA kernels (``vlmrl._C``) with PyTorch oracles.

Every public function dispatches on the device of its first tensor argument:
CUDA tensors run the native kernel (and raise if the extension is not built —
there is no silent fallback on a GPU), CPU tensors run the fp32 oracle in
``vlmrl.ops.reference`` (the CPU/gloo test path).  Shapes and layouts are
documented in ``vlmrl.ops.reference``.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from vlmrl.ops import reference as ref
from vlmrl.ops._ext import ext, has_ext

# GEMM epilogue codes (must match csrc/gemm_sm100.cu)
EPI_STORE = 0
EPI_SWIGLU = 1
EPI_SWIGLU_BWD = 6
EPI_GELU_TANH = 2
EPI_GELU_ERF = 3


def launch_count() -> int:
    """Kernel launches issued by the native library so far (0 when it is not loaded)."""
    return int(ext().launch_count()) if has_ext() else 0


class static_weights:
    """Context: parameters are read-only inside (decode loop), so GEMMs may stream weights ahead of their
    dependency wait (programmatic dependent launch).  Never use it around optimizer or collective updates."""

    def __enter__(self):
        if has_ext():
            ext().set_static_weights(True)
        return self

    def __exit__(self, *exc):
        if has_ext():
            ext().set_static_weights(False)
        return False


class KernelTimeout(RuntimeError):
    """A bounded wait inside a kernel ran out (a pipeline stage never completed); the kernel left without
    touching its outputs and the CUDA context is still usable."""

    def __init__(self, code: int, device: int, what: str):
        super().__init__(f"vlmrl kernel error {code} ({what}) on cuda:{device}")
        self.code = code
        self.device = device


class CollectiveTimeout(KernelTimeout):
    """A peer-memory collective waited longer than its budget for another rank's signal (the rank is
    dead, hung or has left the step)."""


_ERR_WHAT = {1: "TMA producer wait timed out", 2: "MMA wait timed out", 3: "epilogue wait timed out",
             4: "peer rank signal timed out", 5: "bad arguments", 6: "pipeline flag wait timed out",
             7: "gathered weight chunk never arrived"}


def check_errors(device: Optional[int] = None) -> None:
    """Raise ``KernelTimeout`` / ``CollectiveTimeout`` if a kernel recorded an error (reads and clears the
    device error word; synchronises the current stream)."""
    if not has_ext() or not torch.cuda.is_available():
        return
    dev = torch.cuda.current_device() if device is None else int(device)
    code = int(ext().read_and_clear_error(dev))
    if code:
        cls = CollectiveTimeout if code == 4 else KernelTimeout
        raise cls(code, dev, _ERR_WHAT.get(code, "unknown"))


def _cuda(x: torch.Tensor) -> bool:
    return x.is_cuda


class ShardedWeight:
    """A weight matrix whose rows are spread over the ranks' shards of a flat parameter unit.

    ``local`` is the matrix's view inside this rank's copy of the unit (which starts at ``dst_base``);
    rank r's shard of ``shard_bytes`` bytes is at address ``srcs[r]`` (a peer mapping for the other
    ranks).  A GEMM that receives a ``ShardedWeight`` as B copies the rows from the shards into
    ``local`` inside the kernel while its MMAs run (``flags``/``ctr``: the kernel's zeroed arrival
    counters, one pair per concurrently used weight).  After that GEMM, ``local`` holds the matrix.
    """

    __slots__ = ("local", "srcs", "dst_base", "shard_bytes", "flags", "ctr")

    def __init__(self, local: torch.Tensor, srcs: Sequence[int], dst_base: int, shard_bytes: int,
                 flags: torch.Tensor, ctr: torch.Tensor):
        self.local, self.srcs, self.dst_base, self.shard_bytes = local, list(srcs), int(dst_base), int(shard_bytes)
        self.flags, self.ctr = flags, ctr

    @property
    def shape(self):
        return self.local.shape

    @property
    def dtype(self):
        return self.local.dtype

    @property
    def device(self):
        return self.local.device

    @property
    def is_cuda(self) -> bool:
        return self.local.is_cuda


def _gemm_launch(a, b, d, bias, residual, aux, a_kmajor, b_kmajor, alpha, epi, accumulate):
    if isinstance(b, ShardedWeight):
        ext().gemm_gather(a, b.local, d, bias, residual, aux, a_kmajor, b_kmajor, alpha, epi, accumulate, b.srcs,
                          b.dst_base, b.shard_bytes, b.flags, b.ctr)
    else:
        ext().gemm(a, b, d, bias, residual, aux, a_kmajor, b_kmajor, alpha, epi, accumulate)


def unit_gather(srcs: Sequence[int], dst_base: int, shard_bytes: int, ranges: Sequence[Tuple[int, int]]) -> None:
    """Copy byte ranges of a sharded flat unit from every rank's shard into the local copy (CUDA only)."""
    for i in range(0, len(ranges), 8):
        part = ranges[i:i + 8]
        ext().unit_gather(list(srcs), int(dst_base), int(shard_bytes), [int(a) for a, _ in part],
                          [int(b) for _, b in part])


def _opt(x: Optional[torch.Tensor]):
    return x if x is not None else torch.Tensor()


# ------------------------------------------------------------------ GEMM family
def gemm(a: torch.Tensor, b: torch.Tensor, *, a_kmajor: bool = True, b_kmajor: bool = True,
         bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None, alpha: float = 1.0,
         out_dtype: torch.dtype = torch.bfloat16, accumulate: Optional[torch.Tensor] = None,
         out: Optional[torch.Tensor] = None, epilogue: int = EPI_STORE,
         aux: Optional[torch.Tensor] = None) -> torch.Tensor:
    """D = alpha * A·Bᵀ (+bias)(+residual)(+=accumulate) with an optional activation epilogue.

    ``epilogue=EPI_SWIGLU`` treats column pairs (2j, 2j+1) as (gate, up) and
    writes ``silu(gate)*up`` into an ``[M, N/2]`` output; ``aux`` (optional
    ``[M, N]``) then receives the pre-activation.
    """
    M = a.shape[0] if a_kmajor else a.shape[1]
    N = b.shape[0] if b_kmajor else b.shape[1]
    if not _cuda(a):
        if epilogue == EPI_SWIGLU:
            pre = ref.gemm(a, b, a_kmajor=a_kmajor, b_kmajor=b_kmajor, bias=bias, alpha=alpha, out_dtype=torch.float32)
            if aux is not None:
                aux.copy_(pre.to(aux.dtype))
            res = ref.swiglu_interleaved(pre).to(out_dtype)
        elif epilogue in (EPI_GELU_TANH, EPI_GELU_ERF):
            pre = ref.gemm(a, b, a_kmajor=a_kmajor, b_kmajor=b_kmajor, bias=bias, alpha=alpha, out_dtype=torch.float32)
            res = ref.gelu(pre, "tanh" if epilogue == EPI_GELU_TANH else "none").to(out_dtype)
        else:
            res = ref.gemm(a, b, a_kmajor=a_kmajor, b_kmajor=b_kmajor, bias=bias, residual=residual, alpha=alpha,
                           out_dtype=out_dtype, accumulate=accumulate)
        if out is not None and accumulate is None:
            out.copy_(res)
            return out
        return res
    if accumulate is not None:
        d = accumulate
    elif out is not None:
        d = out
    else:
        width = N // 2 if epilogue == EPI_SWIGLU else N
        d = torch.empty(M, width, dtype=out_dtype, device=a.device)
    _gemm_launch(a, b, d, _opt(bias), _opt(residual), _opt(aux), bool(a_kmajor), bool(b_kmajor), float(alpha),
                 int(epilogue), accumulate is not None)
    return d


def linear(x: torch.Tensor, w: torch.Tensor, bias=None, residual=None, out_dtype=torch.bfloat16, out=None):
    """y = x @ w.T (+ bias) (+ residual)."""
    return gemm(x, w, bias=bias, residual=residual, out_dtype=out_dtype, out=out)


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, save_pre: bool = True):
    """act [M,F] = silu(gate)*up for interleaved w_gu [2F,K]; also returns pre [M,2F] when ``save_pre``."""
    pre = torch.empty(x.shape[0], w_gu.shape[0], dtype=x.dtype, device=x.device) if save_pre else None
    act = gemm(x, w_gu, epilogue=EPI_SWIGLU, aux=pre, out_dtype=x.dtype)
    return act, pre


def gemm_partials(a: torch.Tensor, b: torch.Tensor):
    """Stream-K partial sums of ``a @ b.T`` for the fused decode consumers: (ws fp32 [slots, M, N], meta).

    CUDA only: the CPU executor never takes the fused decode path.
    """
    return ext().gemm_partials(a, b)


def dec_qkv(ws, meta, bias, q_w, k_w, lengths, delta, rope: "RopeCfg", k_cache, v_cache, *, n_q: int, n_kv: int,
            eps: float, prefetch=None, block_table=None):
    """Sum QKV partials (+bias), RMSNorm q/k heads (skipped when ``q_w`` is None), MRoPE at position
    ``lengths + delta``, write k/v into the cache at ``lengths``; returns q [B, n_q, D].

    ``prefetch`` (here and in the other decode consumers): a weight tensor whose bytes every CTA asks the
    L2 to fetch while the kernel runs, so the next GEMM streams it from L2.  ``block_table``: the cache
    layer is a block pool (``paged_rows``)."""
    f, _ = rope.device_tables(ws.device)
    return ext().dec_qkv(ws, list(meta), _opt(bias), _opt(q_w), _opt(k_w), lengths, delta, f, k_cache, v_cache, n_q, n_kv,
                         float(eps), prefetch, block_table)


def dec_linear_qkv(x, w, bias, q_w, k_w, lengths, delta, rope: "RopeCfg", k_cache, v_cache, *, n_q: int, n_kv: int,
                   eps: float):
    """``dec_qkv`` of ``x @ w.T`` in one launch: the consumer runs inside the stream-K GEMM after a grid-wide
    barrier (CUDA only)."""
    f, _ = rope.device_tables(x.device)
    return ext().dec_gemm_qkv(x, w, _opt(bias), _opt(q_w), _opt(k_w), lengths, delta, f, k_cache, v_cache, n_q, n_kv,
                              float(eps))


def dec_linear_residual_norm(x, w, residual, nw, eps: float):
    """``dec_residual_norm`` of ``x @ w.T`` in one launch (consumer fused into the GEMM; CUDA only)."""
    return ext().dec_gemm_residual_norm(x, w, residual, nw, float(eps))


def dec_linear_swiglu(x, w):
    """``dec_swiglu`` of ``x @ w.T`` in one launch (consumer fused into the GEMM; CUDA only)."""
    return ext().dec_gemm_swiglu(x, w)


def dec_residual_norm(ws, meta, residual, w, eps: float, prefetch=None):
    """h = sum(partials) + residual (bf16); returns (h, rms_norm(h) * w)."""
    return ext().dec_residual_norm(ws, list(meta), residual, w, float(eps), prefetch)


def dec_swiglu(ws, meta, prefetch=None):
    """silu(gate) * up of interleaved gate/up partial sums -> [M, N/2] bf16."""
    return ext().dec_swiglu(ws, list(meta), prefetch)


def grad_input(dy: torch.Tensor, w: torch.Tensor, out_dtype=torch.bfloat16, out=None):
    """dX [M,K] = dY [M,N] @ W [N,K]."""
    return gemm(dy, w, b_kmajor=False, out_dtype=out_dtype, out=out)


def grad_input_swiglu(dy: torch.Tensor, w_down: torch.Tensor, pre: torch.Tensor):
    """d pre [M, 2F] (interleaved gate/up) of ``act = silu(gate) * up`` given dL/d(act @ w_down.T) = dy.

    On the GPU the down-projection dgrad GEMM applies the SwiGLU backward in its epilogue, so dL/d act is
    never written to memory.
    """
    if not _cuda(dy):
        return swiglu_bwd(grad_input(dy, w_down, out_dtype=dy.dtype), pre)
    M, F = dy.shape[0], w_down.shape[1]
    out = torch.empty(M, 2 * F, dtype=torch.bfloat16, device=dy.device)
    _gemm_launch(dy, w_down, out, torch.Tensor(), torch.Tensor(), pre, True, False, 1.0, EPI_SWIGLU_BWD, False)
    return out


def grad_weight(dy: torch.Tensor, x: torch.Tensor, accumulate: Optional[torch.Tensor] = None,
                out_dtype=torch.float32):
    """dW [N,K] (+)= dY[M,N]ᵀ @ X[M,K] (fp32 accumulation buffer)."""
    return gemm(dy, x, a_kmajor=False, b_kmajor=False, out_dtype=out_dtype, accumulate=accumulate)


def swiglu_bwd(d_act: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    if not _cuda(d_act):
        return ref.swiglu_bwd(d_act, pre)
    out = torch.empty_like(pre)
    ext().swiglu_bwd(d_act, pre, out)
    return out


# ------------------------------------------------------------------ norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    if not _cuda(x):
        return ref.rms_norm(x, w, eps)
    y = torch.empty_like(x)
    rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    ext().rms_norm_fwd(x, w, y, rstd, float(eps))
    return y, rstd


def rms_norm_bwd(dy, x, w, rstd, dw_accum: Optional[torch.Tensor] = None, add: Optional[torch.Tensor] = None):
    """Returns dx (+ ``add``, a second gradient of the same tensor, summed before rounding); adds the weight
    gradient into ``dw_accum`` (fp32 [H]) when given."""
    if not _cuda(x):
        dx, dw = ref.rms_norm_bwd(dy, x, w, rstd)
        if dw_accum is not None:
            dw_accum.add_(dw.to(dw_accum.dtype))
        if add is not None:
            dx = (dx.float() + add.float()).to(dx.dtype)
        return dx
    dx = torch.empty_like(x)
    ext().rms_norm_bwd(dy, x, w, rstd, dx, _opt(dw_accum), _opt(add))
    return dx


def layer_norm(x, w, b, eps: float):
    if not _cuda(x):
        return ref.layer_norm(x, w, b, eps)
    y = torch.empty_like(x)
    ext().layer_norm_fwd(x, w, _opt(b), y, float(eps))
    return y


# ------------------------------------------------------------------ rotary
class RopeCfg:
    """Static rotary parameters of a text decoder (head_dim, theta, MRoPE sections, layout)."""

    def __init__(self, head_dim: int, theta: float, section: Sequence[int], interleaved: bool):
        self.head_dim = int(head_dim)
        self.theta = float(theta)
        self.section = tuple(int(s) for s in section)
        self.interleaved = bool(interleaved)
        self._tables = {}

    def device_tables(self, device) -> Tuple[torch.Tensor, torch.Tensor]:
        """(inv_freq fp32 [D/2], axis int32 [D/2]) resident on ``device``."""
        key = str(device)
        if key not in self._tables:
            from vlmrl.models.qwen3vl.rope import inv_freq, mrope_axis_map

            f = torch.from_numpy(inv_freq(self.head_dim, self.theta)).to(device)
            a = torch.from_numpy(mrope_axis_map(self.section, self.head_dim // 2, self.interleaved)).to(device)
            self._tables[key] = (f, a.to(torch.int32))
        return self._tables[key]


def qk_norm_rope(qkv, q_w, k_w, pos, rope: RopeCfg, *, n_q: int, n_kv: int, eps: float):
    if not _cuda(qkv):
        return ref.qk_norm_rope(qkv, q_w, k_w, pos, n_q=n_q, n_kv=n_kv, head_dim=rope.head_dim, theta=rope.theta,
                                section=rope.section, interleaved=rope.interleaved, eps=eps)
    T, D = qkv.shape[0], rope.head_dim
    q = torch.empty(T, n_q, D, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty(T, n_kv, D, dtype=qkv.dtype, device=qkv.device)
    v = torch.empty(T, n_kv, D, dtype=qkv.dtype, device=qkv.device)
    rq = torch.empty(T, n_q, dtype=torch.float32, device=qkv.device)
    rk = torch.empty(T, n_kv, dtype=torch.float32, device=qkv.device)
    f, ax = rope.device_tables(qkv.device)
    ext().qk_norm_rope_fwd(qkv, _opt(q_w), _opt(k_w), pos, f, ax, q, k, v, rq, rk, n_q, n_kv, float(eps))
    return q, k, v, rq, rk


def qk_norm_rope_bwd(dq, dk, dv, qkv, q_w, k_w, pos, rq, rk, rope: RopeCfg, *, n_q, n_kv, eps,
                     dqw_accum=None, dkw_accum=None):
    if not _cuda(qkv):
        dqkv, dqw, dkw = ref.qk_norm_rope_bwd(dq, dk, dv, qkv, q_w, k_w, pos, rq, rk, n_q=n_q, n_kv=n_kv,
                                              head_dim=rope.head_dim, theta=rope.theta, section=rope.section,
                                              interleaved=rope.interleaved, eps=eps)
        if dqw_accum is not None and dqw is not None:
            dqw_accum.add_(dqw)
        if dkw_accum is not None and dkw is not None:
            dkw_accum.add_(dkw)
        return dqkv
    dqkv = torch.empty_like(qkv)
    f, ax = rope.device_tables(qkv.device)
    ext().qk_norm_rope_bwd(dq, dk, dv, qkv, _opt(q_w), _opt(k_w), pos, f, ax, rq, rk, dqkv, _opt(dqw_accum),
                           _opt(dkw_accum),
                           n_q, n_kv, float(eps))
    return dqkv


def vision_rope(qkv, rc, *, n_heads: int, head_dim: int, style: int = 0):
    """ViT 2-D rotary; ``style`` 0 is HF's pairing, 1 the reference tower's (see ``reference.vision_rope``)."""
    if not _cuda(qkv):
        return ref.vision_rope(qkv, rc, n_heads=n_heads, head_dim=head_dim, style=style)
    N = qkv.shape[0]
    q = torch.empty(N, n_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    ext().vision_rope(qkv, rc, q, k, v, n_heads, int(style))
    return q, k, v


# ------------------------------------------------------------------ attention
_ATTN_DIMS = (16, 32, 64, 128)


def flash_attn(q, k, v, cu_seqlens, max_seqlen: int, *, causal: bool, scale: Optional[float] = None, pre=None):
    """Varlen GQA attention; ``pre`` (int32 [segments, 2]) adds a shared, unmasked key prefix per segment."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not _cuda(q):
        return ref.flash_attn(q, k, v, cu_seqlens, max_seqlen, causal=causal, scale=scale, pre=pre)
    D = q.shape[-1]
    if D not in _ATTN_DIMS:
        # head sizes without a kernel instance (e.g. 80 in the Qwen2.5 ViT): zero-pad to the next one;
        # zero columns add nothing to q.k and produce zero output columns
        Dp = next(d for d in _ATTN_DIMS if d > D)
        pad = lambda t: torch.nn.functional.pad(t, (0, Dp - D)).contiguous()
        o, lse = flash_attn(pad(q), pad(k), pad(v), cu_seqlens, max_seqlen, causal=causal, scale=scale, pre=pre)
        return o[..., :D].contiguous(), lse
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    ext().flash_attn_fwd(q, k, v, cu_seqlens, o, lse, int(max_seqlen), bool(causal), float(scale), pre)
    return o, lse


def flash_attn_bwd(do, q, k, v, o, lse, cu_seqlens, max_seqlen: int, *, causal: bool, scale: Optional[float] = None,
                   pre=None, xq=None):
    """Backward of ``flash_attn``; with ``pre`` also ``xq`` [segments, 2]: the query rows outside each
    segment that attend to all of its keys (the inverse map of ``pre``)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not _cuda(q):
        return ref.flash_attn_bwd(do, q, k, v, o, lse, cu_seqlens, max_seqlen, causal=causal, scale=scale, pre=pre)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    ext().flash_attn_bwd(do, q, k, v, o, lse, cu_seqlens, dq, dk, dv, int(max_seqlen), bool(causal), float(scale),
                         pre, xq)
    return dq, dk, dv


def decode_attn(q, k_cache, v_cache, lengths, *, scale: Optional[float] = None, out=None, prefetch=None,
                lead=None, share_len=None, block_table=None):
    """``prefetch``: a weight the L2 should fetch while the kernel runs (the next GEMM's operand).
    ``lead``/``share_len`` (int32 [B]): the first ``share_len[b]`` cache entries of row b equal those of row
    ``lead[b]`` (members of a GRPO group share the prompt); the kernel then reads them from the leader's
    row, so a group streams its prompt's KV once.  ``block_table`` (int32 [B, blocks]): the caches are
    block pools [NB, Hkv, 64, D] and row b's token t lives in block ``block_table[b, t // 64]``."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not _cuda(q):
        if block_table is not None:
            k_cache, v_cache = paged_rows(k_cache, block_table), paged_rows(v_cache, block_table)
        return ref.decode_attn(q, k_cache, v_cache, lengths, scale=scale)
    o = out if out is not None else torch.empty_like(q)
    ext().decode_attn(q, k_cache, v_cache, lengths, o, float(scale), prefetch, lead, share_len, block_table)
    return o


KV_BLOCK = 64   # tokens per block of a paged KV cache (kv_layout.cuh)


def paged_rows(pool, block_table):
    """The contiguous view [B, Hkv, blocks * 64, D] of a block pool [NB, Hkv, 64, D] under ``block_table``
    (a gathered copy; for host-side consumers and the CPU executor)."""
    B, nb = block_table.shape
    g = pool[block_table.long().reshape(-1)]                       # [B * nb, Hkv, 64, D]
    return g.view(B, nb, pool.shape[1], KV_BLOCK, pool.shape[3]).permute(0, 2, 1, 3, 4).reshape(
        B, pool.shape[1], nb * KV_BLOCK, pool.shape[3])


def kv_write(k, v, k_cache, v_cache, seq_idx, pos_idx, block_table=None):
    """Scatter packed k, v [T,Hkv,D] into caches [B,Hkv,Tmax,D] at (seq_idx[t], pos_idx[t]); with
    ``block_table`` the caches are block pools [NB, Hkv, 64, D]."""
    if not _cuda(k):
        si, pi = seq_idx.long(), pos_idx.long()
        if block_table is not None:
            si = block_table.long()[si, pi // KV_BLOCK]
            pi = pi % KV_BLOCK
        k_cache[si, :, pi] = k.to(k_cache.dtype)
        v_cache[si, :, pi] = v.to(v_cache.dtype)
        return
    ext().kv_write(k, v, k_cache, v_cache, seq_idx, pos_idx, block_table)


# ------------------------------------------------------------------ embedding
def embed(tokens, table, out=None):
    if not _cuda(table):
        return ref.embed(tokens, table)
    o = out if out is not None else torch.empty(tokens.shape[0], table.shape[1], dtype=table.dtype, device=table.device)
    ext().embed(tokens, table, o)
    return o


def scatter_rows_(h, rows, src, add: bool):
    """In place: h[rows] = src (or += src)."""
    if not _cuda(h):
        h.copy_(ref.scatter_rows(h, rows, src, add))
        return h
    ext().scatter_rows(h, rows, src, bool(add))
    return h


def embed_bwd(tokens, dh, dtable):
    if not _cuda(dh):
        return ref.embed_bwd(tokens, dh, dtable)
    ext().embed_bwd(tokens, dh, dtable)
    return dtable


# ------------------------------------------------------------------ vocab
def vocab_logprob(h, w, targets):
    """(logp[target], entropy, lse) fp32 [M] without materialising fp32 logits."""
    if not _cuda(h):
        return ref.vocab_logprob(h, w, targets)
    M = h.shape[0]
    logp = torch.empty(M, dtype=torch.float32, device=h.device)
    ent = torch.empty_like(logp)
    lse = torch.empty_like(logp)
    ext().vocab_logprob_fwd(h, w, targets, logp, ent, lse)
    return logp, ent, lse


def vocab_logprob_bwd(h, w, targets, lse, ent, g_logp, g_ent, dw_accum: torch.Tensor):
    """Returns dh (h.dtype); accumulates dW into ``dw_accum`` (fp32 [V,H])."""
    if not _cuda(h):
        dh, dw = ref.vocab_logprob_bwd(h, w, targets, lse, ent, g_logp, g_ent)
        dw_accum.add_(dw)
        return dh.to(h.dtype)
    dh = torch.empty_like(h)
    ext().vocab_logprob_bwd(h, w, targets, lse, ent, g_logp, g_ent, dh, dw_accum)
    return dh


def lm_logits(h, w, out=None):
    if not _cuda(h):
        return ref.lm_logits(h, w)
    return gemm(h, w, out_dtype=torch.float32, out=out)


# ------------------------------------------------------------------ sampling
def sample(logits, *, temperature: float, top_k: int, top_p: float, seed, step, row_offset: int = 0,
           out_tokens=None, out_logprobs=None):
    """Fused top-k / top-p / temperature sampler.

    ``seed`` and ``step`` may be ints or 1-element int64 CUDA tensors (device
    counters keep a captured CUDA graph valid across replays).
    """
    if not _cuda(logits):
        s = int(step.item()) if torch.is_tensor(step) else int(step)
        sd = int(seed.item()) if torch.is_tensor(seed) else int(seed)
        return ref.sample(logits, temperature=temperature, top_k=top_k, top_p=top_p, seed=sd, step=s,
                          row_offset=row_offset)
    B = logits.shape[0]
    tok = out_tokens if out_tokens is not None else torch.empty(B, dtype=torch.int64, device=logits.device)
    lp = out_logprobs if out_logprobs is not None else torch.empty(B, dtype=torch.float32, device=logits.device)
    if not torch.is_tensor(step):
        step = torch.tensor([int(step)], dtype=torch.int64, device=logits.device)
    if not torch.is_tensor(seed):
        seed = torch.tensor([int(seed) & ((1 << 63) - 1)], dtype=torch.int64, device=logits.device)
    ext().sample(logits, tok, lp, step, seed, float(temperature), int(top_k or 0), float(top_p or 0.0),
                 int(row_offset))
    return tok, lp


FUSED_SAMPLER_MAX_TOPK = 16


def lm_head_sample(h, w, *, temperature: float, top_k: int, top_p: float, seed, step, row_offset: int = 0,
                   out_tokens=None, out_logprobs=None):
    """``sample(h @ w.T, ...)`` without materialising the logits (CUDA, 1 <= top_k <= 16): the lm_head GEMM keeps
    each row's top-k per 128-column tile, a per-row kernel merges them and draws exactly as ``sample`` does."""
    B = h.shape[0]
    tok = out_tokens if out_tokens is not None else torch.empty(B, dtype=torch.int64, device=h.device)
    lp = out_logprobs if out_logprobs is not None else torch.empty(B, dtype=torch.float32, device=h.device)
    if not torch.is_tensor(step):
        step = torch.tensor([int(step)], dtype=torch.int64, device=h.device)
    if not torch.is_tensor(seed):
        seed = torch.tensor([int(seed) & ((1 << 63) - 1)], dtype=torch.int64, device=h.device)
    ext().lm_head_sample(h, w, tok, lp, step, seed, float(temperature), int(top_k), float(top_p or 0.0),
                         int(row_offset))
    return tok, lp


# ------------------------------------------------------------------ optimizer
def adamw_(p, g, m, v, *, lr, beta1, beta2, eps, weight_decay, step, grad_scale=1.0, p_half=None):
    if not _cuda(p):
        return ref.adamw_(p, g, m, v, lr=lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay, step=step,
                          grad_scale=grad_scale, p_half=p_half)
    if torch.is_tensor(grad_scale):
        scale_t = grad_scale
    else:
        scale_t = torch.tensor([float(grad_scale)], dtype=torch.float32, device=p.device)
    ext().adamw(p, g, m, v, _opt(p_half), scale_t, float(lr), float(beta1), float(beta2), float(eps),
                float(weight_decay), int(step))


def sq_norm(x, out: Optional[torch.Tensor] = None):
    """Sum of squares in fp32; with ``out`` ([1] fp32) the result is added into it."""
    if not _cuda(x):
        r = ref.sq_norm(x)
        if out is not None:
            out.add_(r)
            return out
        return r
    o = out if out is not None else torch.zeros(1, dtype=torch.float32, device=x.device)
    ext().sq_norm_acc(x, o)
    return o


def patchify_uint8(images, *, patch: int, temporal: int, merge: int, mean, std, out_dtype=torch.bfloat16):
    if not _cuda(images):
        return ref.patchify_uint8(images, patch=patch, temporal=temporal, merge=merge, mean=mean, std=std).to(out_dtype)
    N, H, W, C = images.shape
    rows = N * (H // patch) * (W // patch)
    out = torch.empty(rows, C * temporal * patch * patch, dtype=out_dtype, device=images.device)
    ms = torch.tensor(list(mean) + list(std), dtype=torch.float32, device=images.device)
    ext().patchify(images, ms, out, patch, temporal, merge)
    return out


__all__ = [n for n in dir() if not n.startswith("_")]
