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
        units.append(UnitLayout(f"layer{i}", [
            ParamSpec("input_norm", (H,), "ones"),
            ParamSpec("qkv_w", (qkv, H)),
            ParamSpec("qkv_b", (qkv,), "zeros"),
            ParamSpec("q_norm", (D,), "ones"),
            ParamSpec("k_norm", (D,), "ones"),
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


def units_to_flax(spec: Qwen3VLSpec, units: Dict[str, torch.Tensor]) -> Dict[str, Any]:
    """Flat unit buffers -> nested dict of fp32 NumPy arrays with Flax names/[in,out] kernels."""
    t = spec.text
    D, nq, nkv = t.head_dim, t.num_attention_heads, t.num_key_value_heads
    tree: Dict[str, Any] = {}
    lays = {l.name: l for l in all_layouts(spec)}
    e = lays["embed"].views(units["embed"])
    _set(tree, "embed/embedding", _np(e["embed"]))
    for i in range(t.num_hidden_layers):
        w = lays[f"layer{i}"].views(units[f"layer{i}"])
        p = f"layers_{i}"
        q_rows, kv_rows = nq * D, nkv * D
        qkv_w, qkv_b = w["qkv_w"], w["qkv_b"]
        for name, a, b in (("q_proj", 0, q_rows), ("k_proj", q_rows, q_rows + kv_rows),
                           ("v_proj", q_rows + kv_rows, q_rows + 2 * kv_rows)):
            _set(tree, f"{p}/attn/{name}/kernel", _np(qkv_w[a:b].t()))
            _set(tree, f"{p}/attn/{name}/bias", _np(qkv_b[a:b]))
        _set(tree, f"{p}/attn/q_norm/weight", _np(w["q_norm"]))
        _set(tree, f"{p}/attn/k_norm/weight", _np(w["k_norm"]))
        _set(tree, f"{p}/attn/o_proj/kernel", _np(w["o_w"].t()))
        _set(tree, f"{p}/mlp/gate_proj/kernel", _np(w["gu_w"][0::2].t()))
        _set(tree, f"{p}/mlp/up_proj/kernel", _np(w["gu_w"][1::2].t()))
        _set(tree, f"{p}/mlp/down_proj/kernel", _np(w["down_w"].t()))
        _set(tree, f"{p}/input_norm/weight", _np(w["input_norm"]))
        _set(tree, f"{p}/post_norm/weight", _np(w["post_norm"]))
    h = lays["head"].views(units["head"])
    _set(tree, "final_norm/weight", _np(h["final_norm"]))
    _set(tree, "lm_head/kernel", _np(h["lm_head"].t()))
    if spec.vision is not None and "visual" in units:
        v = lays["visual"].views(units["visual"])
        _set(tree, "visual/patch_embed/proj/kernel", _np(v["patch_w"].t()))
        _set(tree, "visual/patch_embed/proj/bias", _np(v["patch_b"]))
        if "pos_embed" in v:
            _set(tree, "visual/pos_embed/embedding", _np(v["pos_embed"]))
        for j in range(spec.vision.depth):
            b, p = f"b{j}.", f"visual/blocks_{j}"
            for src, dst in (("n1", "norm1"), ("n2", "norm2")):
                _set(tree, f"{p}/{dst}/weight", _np(v[b + src + "_w"]))
                _set(tree, f"{p}/{dst}/bias", _np(v[b + src + "_b"]))
            for src, dst in (("qkv", "attn/qkv"), ("proj", "attn/proj"), ("fc1", "mlp/linear_fc1"), ("fc2", "mlp/linear_fc2")):
                _set(tree, f"{p}/{dst}/kernel", _np(v[b + src + "_w"].t()))
                _set(tree, f"{p}/{dst}/bias", _np(v[b + src + "_b"]))
        for b, p in _merged_names(spec):
            _set(tree, f"{p}/norm/weight", _np(v[b + "norm_w"]))
            _set(tree, f"{p}/norm/bias", _np(v[b + "norm_b"]))
            for src, dst in (("fc1", "linear1"), ("fc2", "linear2")):
                _set(tree, f"{p}/{dst}/kernel", _np(v[b + src + "_w"].t()))
                _set(tree, f"{p}/{dst}/bias", _np(v[b + src + "_b"]))
    return tree


def flax_to_units(spec: Qwen3VLSpec, tree: Dict[str, Any], dtype=torch.float32, device="cpu",
                  strict: bool = False) -> Dict[str, torch.Tensor]:
    """Nested Flax-named tree -> flat unit buffers.  Missing leaves keep their random init unless ``strict``."""
    units = init_params(spec, seed=0, dtype=dtype, device=device)
    lays = {l.name: l for l in all_layouts(spec)}
    missing: List[str] = []

    def fetch(path: str):
        try:
            return torch.as_tensor(np.asarray(_get(tree, path)), dtype=torch.float32)
        except (KeyError, TypeError):
            missing.append(path)
            return None

    def put(view: torch.Tensor, path: str, transpose: bool = False):
        val = fetch(path)
        if val is None:
            return
        val = val.t() if transpose else val
        if tuple(val.shape) != tuple(view.shape):
            raise ValueError(f"{path}: shape {tuple(val.shape)} != expected {tuple(view.shape)}")
        view.copy_(val.to(view.dtype))

    t = spec.text
    D, nq, nkv = t.head_dim, t.num_attention_heads, t.num_key_value_heads
    put(lays["embed"].views(units["embed"])["embed"], "embed/embedding")
    for i in range(t.num_hidden_layers):
        w = lays[f"layer{i}"].views(units[f"layer{i}"])
        p = f"layers_{i}"
        q_rows, kv_rows = nq * D, nkv * D
        for name, a, b in (("q_proj", 0, q_rows), ("k_proj", q_rows, q_rows + kv_rows),
                           ("v_proj", q_rows + kv_rows, q_rows + 2 * kv_rows)):
            put(w["qkv_w"][a:b], f"{p}/attn/{name}/kernel", True)
            put(w["qkv_b"][a:b], f"{p}/attn/{name}/bias")
        put(w["q_norm"], f"{p}/attn/q_norm/weight")
        put(w["k_norm"], f"{p}/attn/k_norm/weight")
        put(w["o_w"], f"{p}/attn/o_proj/kernel", True)
        put(w["gu_w"][0::2], f"{p}/mlp/gate_proj/kernel", True)
        put(w["gu_w"][1::2], f"{p}/mlp/up_proj/kernel", True)
        put(w["down_w"], f"{p}/mlp/down_proj/kernel", True)
        put(w["input_norm"], f"{p}/input_norm/weight")
        put(w["post_norm"], f"{p}/post_norm/weight")
    h = lays["head"].views(units["head"])
    put(h["final_norm"], "final_norm/weight")
    put(h["lm_head"], "lm_head/kernel", True)
    if spec.vision is not None:
        v = lays["visual"].views(units["visual"])
        put(v["patch_w"], "visual/patch_embed/proj/kernel", True)
        put(v["patch_b"], "visual/patch_embed/proj/bias")
        if "pos_embed" in v:
            put(v["pos_embed"], "visual/pos_embed/embedding")
        for j in range(spec.vision.depth):
            b, p = f"b{j}.", f"visual/blocks_{j}"
            for src, dst in (("n1", "norm1"), ("n2", "norm2")):
                put(v[b + src + "_w"], f"{p}/{dst}/weight")
                put(v[b + src + "_b"], f"{p}/{dst}/bias")
            for src, dst in (("qkv", "attn/qkv"), ("proj", "attn/proj"), ("fc1", "mlp/linear_fc1"), ("fc2", "mlp/linear_fc2")):
                put(v[b + src + "_w"], f"{p}/{dst}/kernel", True)
                put(v[b + src + "_b"], f"{p}/{dst}/bias")
        for b, p in _merged_names(spec):
            put(v[b + "norm_w"], f"{p}/norm/weight")
            put(v[b + "norm_b"], f"{p}/norm/bias")
            for src, dst in (("fc1", "linear1"), ("fc2", "linear2")):
                put(v[b + src + "_w"], f"{p}/{dst}/kernel", True)
                put(v[b + src + "_b"], f"{p}/{dst}/bias")
    if strict and missing:
        raise KeyError(f"checkpoint is missing {len(missing)} leaves, e.g. {missing[:5]}")
    return units


__all__ = ["ALIGN", "ParamSpec", "UnitLayout", "text_layouts", "vision_layout", "all_layouts", "init_unit_",
           "init_params", "unit_seed", "units_to_flax", "flax_to_units"]
