"""Parameter layout: flat per-unit buffers and the Flax-named checkpoint tree.

Parameters live in *units* — contiguous flat buffers that are the granularity
of FSDP gathering/reduction and of the optimizer:

* ``embed``            — ``embed`` [V, H]
* ``layer{i}``         — ``input_norm`` [H], ``qkv_w`` [(nq+2nkv)·D, H], ``qkv_b`` [(nq+2nkv)·D],
                         ``q_norm`` [D], ``k_norm`` [D], ``o_w`` [H, nq·D], ``post_norm`` [H],
                         ``gu_w`` [2F, H] (gate/up rows interleaved), ``down_w`` [H, F]
* ``head``             — ``final_norm`` [H], ``lm_head`` [V, H]
* ``visual``           — the whole (frozen) vision tower

Every parameter starts on a 256-byte boundary inside its unit (TMA operands
must be 16-byte aligned).  Weights keep the PyTorch ``[out, in]`` layout.

The checkpoint tree is the reference's Flax naming with ``[in, out]`` Dense
kernels (reference ``models/qwen3vl/model.py:987-1086``, transposition at
``:1160-1161``): ``embed/embedding``, ``layers_{i}/attn/{q,k,v}_proj/{kernel,bias}``,
``layers_{i}/attn/{q,k}_norm/weight``, ``layers_{i}/attn/o_proj/kernel``,
``layers_{i}/mlp/{gate,up,down}_proj/kernel``, ``layers_{i}/{input,post}_norm/weight``,
``final_norm/weight``, ``lm_head/kernel``.  HF-faithful vision keys extend the
reference's (``visual/patch_embed/proj/{kernel,bias}``, ``visual/pos_embed/embedding``,
``visual/blocks_{j}/{norm1,norm2}/{weight,bias}``, ``visual/blocks_{j}/attn/{qkv,proj}/{kernel,bias}``,
``visual/blocks_{j}/mlp/linear_fc{1,2}/{kernel,bias}``, ``visual/merger/...``,
``visual/deepstack_mergers_{k}/...`` with ``norm`` and ``linear1``/``linear2``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, List, Optional, Tuple

import numpy as np
import torch

from vlmrl.models.qwen3vl.config import Qwen3VLSpec

ALIGN = 128  # elements (256 bytes in bf16)


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class ParamSpec:
    name: str
    shape: Tuple[int, ...]
    init: str = "normal"      # normal | ones | zeros
    std: float = 0.02

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1


@dataclass
class UnitLayout:
    name: str
    params: List[ParamSpec]
    trainable: bool = True
    offsets: Dict[str, int] = field(default_factory=dict)
    numel: int = 0

    def __post_init__(self):
        off = 0
        for p in self.params:
            self.offsets[p.name] = off
            off = _round_up(off + p.numel, ALIGN)
        self.numel = off

    def spec(self, name: str) -> ParamSpec:
        for p in self.params:
            if p.name == name:
                return p
        raise KeyError(name)

    def views(self, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
        if flat.numel() < self.numel:
            raise ValueError(f"unit {self.name}: buffer has {flat.numel()} < {self.numel} elements")
        return {p.name: flat[self.offsets[p.name]:self.offsets[p.name] + p.numel].view(p.shape) for p in self.params}

    def padded_numel(self, world: int) -> int:
        return _round_up(self.numel, ALIGN * world)


# --------------------------------------------------------------------------- layouts
def text_layouts(spec: Qwen3VLSpec) -> List[UnitLayout]:
    t = spec.text
    H, D, nq, nkv, F, V = t.hidden_size, t.head_dim, t.num_attention_heads, t.num_key_value_heads, t.intermediate_size, t.vocab_size
    qkv = (nq + 2 * nkv) * D
    units = [UnitLayout("embed", [ParamSpec("embed", (V, H))])]
    for i in range(t.num_hidden_layers):
        norms = [ParamSpec("q_norm", (D,), "ones"), ParamSpec("k_norm", (D,), "ones")] if t.qk_norm else []
        units.append(UnitLayout(f"layer{i}", [
            ParamSpec("input_norm", (H,), "ones"),
            ParamSpec("qkv_w", (qkv, H)),
            ParamSpec("qkv_b", (qkv,), "zeros"),
            *norms,
            ParamSpec("o_w", (H, nq * D)),
            ParamSpec("post_norm", (H,), "ones"),
            ParamSpec("gu_w", (2 * F, H)),
            ParamSpec("down_w", (H, F)),
        ]))
    units.append(UnitLayout("head", [ParamSpec("final_norm", (H,), "ones"), ParamSpec("lm_head", (V, H))]))
    return units


def vision_layout(spec: Qwen3VLSpec) -> Optional[UnitLayout]:
    v = spec.vision
    if v is None:
        return None
    Hv, I, out, M = v.hidden_size, v.intermediate_size, v.out_hidden_size, v.merged_hidden_size
    if spec.vision_arch in ("qwen25", "reference"):
        # RMSNorm blocks with a biased SwiGLU MLP (gate/up rows interleaved), RMSNorm merger(s); the
        # reference tower adds one post-shuffle merger (RMSNorm over 4*Hv) per deepstack index
        ps = [ParamSpec("patch_w", (Hv, v.patch_volume))]
        for j in range(v.depth):
            p = f"b{j}."
            ps += [ParamSpec(p + "n1_w", (Hv,), "ones"),
                   ParamSpec(p + "qkv_w", (3 * Hv, Hv)), ParamSpec(p + "qkv_b", (3 * Hv,), "zeros"),
                   ParamSpec(p + "proj_w", (Hv, Hv)), ParamSpec(p + "proj_b", (Hv,), "zeros"),
                   ParamSpec(p + "n2_w", (Hv,), "ones"),
                   ParamSpec(p + "gu_w", (2 * I, Hv)), ParamSpec(p + "gu_b", (2 * I,), "zeros"),
                   ParamSpec(p + "down_w", (Hv, I)), ParamSpec(p + "down_b", (Hv,), "zeros")]
        mergers = [("m.", Hv)]
        if spec.vision_arch == "reference":
            mergers += [(f"d{k}.", M) for k in range(len(v.deepstack_visual_indexes))]
        for prefix, norm_dim in mergers:
            ps += [ParamSpec(prefix + "norm_w", (norm_dim,), "ones"),
                   ParamSpec(prefix + "fc1_w", (M, M)), ParamSpec(prefix + "fc1_b", (M,), "zeros"),
                   ParamSpec(prefix + "fc2_w", (out, M)), ParamSpec(prefix + "fc2_b", (out,), "zeros")]
        return UnitLayout("visual", ps, trainable=False)
    ps = [ParamSpec("patch_w", (Hv, v.patch_volume)), ParamSpec("patch_b", (Hv,), "zeros")]
    if v.num_position_embeddings:
        ps.append(ParamSpec("pos_embed", (int(v.num_position_embeddings), Hv)))
    for j in range(v.depth):
        p = f"b{j}."
        ps += [ParamSpec(p + "n1_w", (Hv,), "ones"), ParamSpec(p + "n1_b", (Hv,), "zeros"),
               ParamSpec(p + "qkv_w", (3 * Hv, Hv)), ParamSpec(p + "qkv_b", (3 * Hv,), "zeros"),
               ParamSpec(p + "proj_w", (Hv, Hv)), ParamSpec(p + "proj_b", (Hv,), "zeros"),
               ParamSpec(p + "n2_w", (Hv,), "ones"), ParamSpec(p + "n2_b", (Hv,), "zeros"),
               ParamSpec(p + "fc1_w", (I, Hv)), ParamSpec(p + "fc1_b", (I,), "zeros"),
               ParamSpec(p + "fc2_w", (Hv, I)), ParamSpec(p + "fc2_b", (Hv,), "zeros")]
    mergers = [("m.", Hv)] + [(f"d{k}.", M) for k in range(len(v.deepstack_visual_indexes))]
    for prefix, norm_dim in mergers:
        ps += [ParamSpec(prefix + "norm_w", (norm_dim,), "ones"), ParamSpec(prefix + "norm_b", (norm_dim,), "zeros"),
               ParamSpec(prefix + "fc1_w", (M, M)), ParamSpec(prefix + "fc1_b", (M,), "zeros"),
               ParamSpec(prefix + "fc2_w", (out, M)), ParamSpec(prefix + "fc2_b", (out,), "zeros")]
    return UnitLayout("visual", ps, trainable=False)


def all_layouts(spec: Qwen3VLSpec) -> List[UnitLayout]:
    units = text_layouts(spec)
    vl = vision_layout(spec)
    if vl is not None:
        units.append(vl)
    return units


# --------------------------------------------------------------------------- init
def init_unit_(layout: UnitLayout, flat: torch.Tensor, seed: int) -> None:
    """Random init of one unit in place: N(0, std) for matrices, ones/zeros for norms and biases.

    Draws come from a generator on ``flat``'s device seeded with ``seed`` (a
    device-side draw keeps multi-GB inits off the host).
    """
    views = layout.views(flat)
    flat.zero_()
    gen = torch.Generator(device=flat.device).manual_seed(int(seed) & 0x7FFFFFFFFFFF)
    for p in layout.params:
        v = views[p.name]
        if p.init == "ones":
            v.fill_(1.0)
        elif p.init == "zeros":
            v.zero_()
        elif v.dtype == torch.float32:
            v.normal_(0.0, p.std, generator=gen)
        else:
            tmp = torch.empty(p.shape, dtype=torch.float32, device=flat.device)
            tmp.normal_(0.0, p.std, generator=gen)
            v.copy_(tmp)
            del tmp


def unit_seed(seed: int, index: int) -> int:
    return (int(seed) * 1000003 + 7919 * int(index)) & 0x7FFFFFFF


def init_params(spec: Qwen3VLSpec, seed: int = 0, dtype=torch.float32, device="cpu",
                units: Optional[Iterable[str]] = None) -> Dict[str, torch.Tensor]:
    """Full (unsharded) flat buffers for every unit, random-initialised from ``seed``.

    A tied model (``tie_word_embeddings``) starts with ``lm_head == embed``;
    afterwards the two are trained independently (reference
    ``models/qwen3vl/model.py:1167-1174``).
    """
    wanted = set(units) if units is not None else None
    out: Dict[str, torch.Tensor] = {}
    lays = all_layouts(spec)
    for i, lay in enumerate(lays):
        if wanted is not None and lay.name not in wanted:
            continue
        buf = torch.empty(lay.numel, dtype=dtype, device=device)
        init_unit_(lay, buf, unit_seed(seed, i))
        out[lay.name] = buf
    if spec.text.tie_word_embeddings and "head" in out and "embed" in out:
        by = {l.name: l for l in lays}
        by["head"].views(out["head"])["lm_head"].copy_(by["embed"].views(out["embed"])["embed"])
    return out


# --------------------------------------------------------------------------- flax tree conversion
def _set(tree: Dict[str, Any], path: str, value) -> None:
    node = tree
    keys = path.split("/")
    for k in keys[:-1]:
        node = node.setdefault(k, {})
    node[keys[-1]] = value


def _get(tree: Dict[str, Any], path: str):
    node = tree
    for k in path.split("/"):
        node = node[k]
    return node


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu", torch.float32).numpy().copy()


def _merged_names(spec: Qwen3VLSpec):
    v = spec.vision
    yield "m.", "visual/merger"
    for k in range(len(v.deepstack_visual_indexes)):
        yield f"d{k}.", f"visual/deepstack_mergers_{k}"


def flax_leaves(spec: Qwen3VLSpec, views: Dict[str, Dict[str, torch.Tensor]]):
    """Yield (Flax path, unit view, transposed) for every leaf of the checkpoint tree.

    Dense kernels are stored ``[in, out]`` (transposed from the unit's ``[out, in]``
    rows); the fused qkv / interleaved gate-up rows are split into the separate
    q/k/v and gate/up leaves.  Both the Qwen3-VL tree and the Qwen2.5-VL tree
    (no q/k norms; RMSNorm + SwiGLU ViT; ``merger/norm`` without bias) are covered.
    """
    t = spec.text
    D, nq, nkv = t.head_dim, t.num_attention_heads, t.num_key_value_heads
    q_rows, kv_rows = nq * D, nkv * D
    yield "embed/embedding", views["embed"]["embed"], False
    for i in range(t.num_hidden_layers):
        w = views[f"layer{i}"]
        p = f"layers_{i}"
        for name, a, b in (("q_proj", 0, q_rows), ("k_proj", q_rows, q_rows + kv_rows),
                           ("v_proj", q_rows + kv_rows, q_rows + 2 * kv_rows)):
            yield f"{p}/attn/{name}/kernel", w["qkv_w"][a:b], True
            yield f"{p}/attn/{name}/bias", w["qkv_b"][a:b], False
        if "q_norm" in w:
            yield f"{p}/attn/q_norm/weight", w["q_norm"], False
            yield f"{p}/attn/k_norm/weight", w["k_norm"], False
        yield f"{p}/attn/o_proj/kernel", w["o_w"], True
        yield f"{p}/mlp/gate_proj/kernel", w["gu_w"][0::2], True
        yield f"{p}/mlp/up_proj/kernel", w["gu_w"][1::2], True
        yield f"{p}/mlp/down_proj/kernel", w["down_w"], True
        yield f"{p}/input_norm/weight", w["input_norm"], False
        yield f"{p}/post_norm/weight", w["post_norm"], False
    yield "final_norm/weight", views["head"]["final_norm"], False
    yield "lm_head/kernel", views["head"]["lm_head"], True
    if spec.vision is None or "visual" not in views:
        return
    v = views["visual"]
    yield "visual/patch_embed/proj/kernel", v["patch_w"], True
    if spec.vision_arch in ("qwen25", "reference"):
        for j in range(spec.vision.depth):
            b, p = f"b{j}.", f"visual/blocks_{j}"
            yield f"{p}/norm1/weight", v[b + "n1_w"], False
            yield f"{p}/norm2/weight", v[b + "n2_w"], False
            for src, dst in (("qkv", "attn/qkv"), ("proj", "attn/proj")):
                yield f"{p}/{dst}/kernel", v[b + src + "_w"], True
                yield f"{p}/{dst}/bias", v[b + src + "_b"], False
            yield f"{p}/mlp/gate_proj/kernel", v[b + "gu_w"][0::2], True
            yield f"{p}/mlp/gate_proj/bias", v[b + "gu_b"][0::2], False
            yield f"{p}/mlp/up_proj/kernel", v[b + "gu_w"][1::2], True
            yield f"{p}/mlp/up_proj/bias", v[b + "gu_b"][1::2], False
            yield f"{p}/mlp/down_proj/kernel", v[b + "down_w"], True
            yield f"{p}/mlp/down_proj/bias", v[b + "down_b"], False
        names = list(_merged_names(spec)) if spec.vision_arch == "reference" else [("m.", "visual/merger")]
        for b, p in names:
            yield f"{p}/norm/weight", v[b + "norm_w"], False
            for src, dst in (("fc1", "linear1"), ("fc2", "linear2")):
                yield f"{p}/{dst}/kernel", v[b + src + "_w"], True
                yield f"{p}/{dst}/bias", v[b + src + "_b"], False
        return
    yield "visual/patch_embed/proj/bias", v["patch_b"], False
    if "pos_embed" in v:
        yield "visual/pos_embed/embedding", v["pos_embed"], False
    for j in range(spec.vision.depth):
        b, p = f"b{j}.", f"visual/blocks_{j}"
        for src, dst in (("n1", "norm1"), ("n2", "norm2")):
            yield f"{p}/{dst}/weight", v[b + src + "_w"], False
            yield f"{p}/{dst}/bias", v[b + src + "_b"], False
        for src, dst in (("qkv", "attn/qkv"), ("proj", "attn/proj"), ("fc1", "mlp/linear_fc1"),
                         ("fc2", "mlp/linear_fc2")):
            yield f"{p}/{dst}/kernel", v[b + src + "_w"], True
            yield f"{p}/{dst}/bias", v[b + src + "_b"], False
    for b, p in _merged_names(spec):
        yield f"{p}/norm/weight", v[b + "norm_w"], False
        yield f"{p}/norm/bias", v[b + "norm_b"], False
        for src, dst in (("fc1", "linear1"), ("fc2", "linear2")):
            yield f"{p}/{dst}/kernel", v[b + src + "_w"], True
            yield f"{p}/{dst}/bias", v[b + src + "_b"], False


def units_to_flax(spec: Qwen3VLSpec, units: Dict[str, torch.Tensor]) -> Dict[str, Any]:
    """Flat unit buffers -> nested dict of fp32 NumPy arrays with Flax names/[in,out] kernels."""
    lays = {l.name: l for l in all_layouts(spec)}
    views = {n: lays[n].views(u) for n, u in units.items() if n in lays}
    tree: Dict[str, Any] = {}
    for path, view, tr in flax_leaves(spec, views):
        _set(tree, path, _np(view.t() if tr else view))
    return tree


def flax_to_units(spec: Qwen3VLSpec, tree: Dict[str, Any], dtype=torch.float32, device="cpu",
                  strict: bool = False) -> Dict[str, torch.Tensor]:
    """Nested Flax-named tree -> flat unit buffers.  Missing leaves keep their random init unless ``strict``."""
    units = init_params(spec, seed=0, dtype=dtype, device=device)
    lays = {l.name: l for l in all_layouts(spec)}
    views = {n: lays[n].views(u) for n, u in units.items()}
    missing: List[str] = []
    for path, view, tr in flax_leaves(spec, views):
        try:
            val = torch.as_tensor(np.asarray(_get(tree, path)), dtype=torch.float32)
        except (KeyError, TypeError):
            missing.append(path)
            continue
        val = val.t() if tr else val
        if tuple(val.shape) != tuple(view.shape):
            raise ValueError(f"{path}: shape {tuple(val.shape)} != expected {tuple(view.shape)}")
        view.copy_(val.to(view.dtype))
    if missing and strict:
        raise KeyError(f"{len(missing)} leaves missing from the params tree, e.g. {missing[:5]}")
    return units

__all__ = ["ALIGN", "ParamSpec", "UnitLayout", "text_layouts", "vision_layout", "all_layouts", "init_unit_",
           "init_params", "unit_seed", "units_to_flax", "flax_to_units"]
