"""HF Qwen3-VL weights <-> flat units, and model construction from HF dirs / checkpoints.

* ``hf_state_dict_to_units`` maps HF tensor names (both the
  ``model.language_model.*`` layout and the older ``model.*`` text layout, with
  or without the extra ``.model`` level) onto the unit layout; the Conv3d patch
  embedding is flattened to ``[Hv, C*Tp*P*P]`` (reference
  ``models/qwen3vl/model.py:1136-1149``); a tied checkpoint without
  ``lm_head.weight`` copies the embedding into ``lm_head``
  (reference ``:1167-1174``).
* ``create_model_from_hf(hf_dir)`` -> (model, Flax-named params tree), the
  converter's entry point (reference ``:1097-1176``).
* ``create_model_from_ckpt(ckpt_dir)`` reads ``config.json`` + ``params.pkl``
  (reference ``:1179-1187``).
"""

from __future__ import annotations

import glob
import json
import os
import re
from typing import Any, Dict, Optional, Tuple

import torch

from vlmrl.models.qwen3vl.config import Qwen3VLSpec, spec_from_config
from vlmrl.models.qwen3vl.params import all_layouts, flax_to_units, init_params, units_to_flax

_TEXT = re.compile(r"^(?:model\.)?(?:language_model\.)?(?:model\.)?")


def _text_key(key: str) -> Optional[str]:
    if "visual." in key:
        return None
    if key.startswith("lm_head."):
        return key
    return _TEXT.sub("", key)


def _vision_key(key: str) -> Optional[str]:
    i = key.find("visual.")
    return key[i + len("visual."):] if i >= 0 else None


def _put_qwen25_vision(v: Dict[str, torch.Tensor], vk: str, val: torch.Tensor, put) -> None:
    """HF Qwen2.5-VL vision tensor names -> the qwen25 ``visual`` unit (gate/up rows interleaved)."""
    m = re.match(r"blocks\.(\d+)\.(.+)\.(weight|bias)$", vk)
    if m:
        j, sub, kind = int(m.group(1)), m.group(2), m.group(3)
        b = f"b{j}."
        if sub in ("norm1", "norm2") and kind == "weight":
            put(v[b + ("n1_w" if sub == "norm1" else "n2_w")], val)
        elif sub in ("attn.qkv", "attn.proj"):
            put(v[b + sub.split(".")[1] + ("_w" if kind == "weight" else "_b")], val)
        elif sub in ("mlp.gate_proj", "mlp.up_proj"):
            rows = slice(0, None, 2) if sub == "mlp.gate_proj" else slice(1, None, 2)
            put(v[b + ("gu_w" if kind == "weight" else "gu_b")][rows], val)
        elif sub == "mlp.down_proj":
            put(v[b + ("down_w" if kind == "weight" else "down_b")], val)
        return
    m = re.match(r"merger\.(ln_q|mlp\.0|mlp\.2)\.(weight|bias)$", vk)
    if m:
        name = {"ln_q": "norm", "mlp.0": "fc1", "mlp.2": "fc2"}[m.group(1)]
        if name == "norm" and m.group(2) == "bias":
            return
        put(v[f"m.{name}_{'w' if m.group(2) == 'weight' else 'b'}"], val)
        return
    # reference tower: HF Qwen3-VL deepstack mergers (LayerNorm bias dropped, as the reference's converter
    # does, reference models/qwen3vl/model.py:1076-1087)
    m = re.match(r"deepstack_merger_list\.(\d+)\.(norm|linear_fc1|linear_fc2)\.(weight|bias)$", vk)
    if m and f"d{int(m.group(1))}.norm_w" in v:
        name = {"norm": "norm", "linear_fc1": "fc1", "linear_fc2": "fc2"}[m.group(2)]
        if name == "norm" and m.group(3) == "bias":
            return
        put(v[f"d{int(m.group(1))}.{name}_{'w' if m.group(3) == 'weight' else 'b'}"], val)


def hf_state_dict_to_units(spec: Qwen3VLSpec, sd: Dict[str, torch.Tensor], dtype=torch.float32,
                           device="cpu") -> Dict[str, torch.Tensor]:
    units = init_params(spec, seed=0, dtype=dtype, device=device)
    lays = {l.name: l for l in all_layouts(spec)}
    t = spec.text
    D, nq, nkv = t.head_dim, t.num_attention_heads, t.num_key_value_heads
    q_rows, kv_rows = nq * D, nkv * D
    views = {n: lays[n].views(units[n]) for n in units}
    seen_lm_head = False

    def put(dst: torch.Tensor, src: torch.Tensor):
        if tuple(dst.shape) != tuple(src.shape):
            raise ValueError(f"shape mismatch {tuple(src.shape)} -> {tuple(dst.shape)}")
        dst.copy_(src.to(dst.dtype))

    for key, val in sd.items():
        val = val.float()
        vk = _vision_key(key)
        if vk is not None and spec.vision is not None:
            v = views["visual"]
            if vk == "patch_embed.proj.weight":
                put(v["patch_w"], val.reshape(val.shape[0], -1))
            elif vk in ("patch_embed.proj.bias", "pos_embed.weight"):
                name = "patch_b" if vk == "patch_embed.proj.bias" else "pos_embed"
                if name in v:  # the RMSNorm towers have neither
                    put(v[name], val)
            elif spec.vision_arch in ("qwen25", "reference"):
                _put_qwen25_vision(v, vk, val, put)
            else:
                m = re.match(r"blocks\.(\d+)\.(.+)\.(weight|bias)$", vk)
                if m:
                    j, sub, kind = int(m.group(1)), m.group(2), "w" if m.group(3) == "weight" else "b"
                    name = {"norm1": "n1", "norm2": "n2", "attn.qkv": "qkv", "attn.proj": "proj",
                            "mlp.linear_fc1": "fc1", "mlp.linear_fc2": "fc2"}.get(sub)
                    if name:
                        put(v[f"b{j}.{name}_{kind}"], val)
                    continue
                m = re.match(r"(merger|deepstack_merger_list\.(\d+))\.(norm|linear_fc1|linear_fc2)\.(weight|bias)$", vk)
                if m:
                    prefix = "m." if m.group(1) == "merger" else f"d{int(m.group(2))}."
                    name = {"norm": "norm", "linear_fc1": "fc1", "linear_fc2": "fc2"}[m.group(3)]
                    put(v[f"{prefix}{name}_{'w' if m.group(4) == 'weight' else 'b'}"], val)
            continue
        tk = _text_key(key)
        if tk is None:
            continue
        if tk == "embed_tokens.weight":
            put(views["embed"]["embed"], val)
        elif tk == "norm.weight":
            put(views["head"]["final_norm"], val)
        elif tk == "lm_head.weight":
            put(views["head"]["lm_head"], val)
            seen_lm_head = True
        else:
            m = re.match(r"layers\.(\d+)\.(.+)$", tk)
            if not m:
                continue
            i, sub = int(m.group(1)), m.group(2)
            w = views[f"layer{i}"]
            slots = {"self_attn.q_proj": (0, q_rows), "self_attn.k_proj": (q_rows, q_rows + kv_rows),
                     "self_attn.v_proj": (q_rows + kv_rows, q_rows + 2 * kv_rows)}
            base, kind = sub.rsplit(".", 1)
            if base in slots:
                a, b = slots[base]
                put(w["qkv_w" if kind == "weight" else "qkv_b"][a:b], val)
            elif sub == "self_attn.o_proj.weight":
                put(w["o_w"], val)
            elif sub == "self_attn.q_norm.weight":
                put(w["q_norm"], val)
            elif sub == "self_attn.k_norm.weight":
                put(w["k_norm"], val)
            elif sub == "mlp.gate_proj.weight":
                put(w["gu_w"][0::2], val)
            elif sub == "mlp.up_proj.weight":
                put(w["gu_w"][1::2], val)
            elif sub == "mlp.down_proj.weight":
                put(w["down_w"], val)
            elif sub == "input_layernorm.weight":
                put(w["input_norm"], val)
            elif sub == "post_attention_layernorm.weight":
                put(w["post_norm"], val)
    if not seen_lm_head:
        views["head"]["lm_head"].copy_(views["embed"]["embed"])
    return units


def units_to_hf_state_dict(spec: Qwen3VLSpec, units: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Units -> HF ``Qwen3VLForConditionalGeneration`` state dict (transformers >= 4.57 naming)."""
    lays = {l.name: l for l in all_layouts(spec)}
    t = spec.text
    D, nq, nkv = t.head_dim, t.num_attention_heads, t.num_key_value_heads
    q_rows, kv_rows = nq * D, nkv * D
    sd: Dict[str, torch.Tensor] = {}
    L = "model.language_model."
    sd[L + "embed_tokens.weight"] = lays["embed"].views(units["embed"])["embed"].clone()
    for i in range(t.num_hidden_layers):
        w = lays[f"layer{i}"].views(units[f"layer{i}"])
        p = f"{L}layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = w["qkv_w"][:q_rows].clone()
        sd[p + "self_attn.k_proj.weight"] = w["qkv_w"][q_rows:q_rows + kv_rows].clone()
        sd[p + "self_attn.v_proj.weight"] = w["qkv_w"][q_rows + kv_rows:].clone()
        if t.attention_bias:
            sd[p + "self_attn.q_proj.bias"] = w["qkv_b"][:q_rows].clone()
            sd[p + "self_attn.k_proj.bias"] = w["qkv_b"][q_rows:q_rows + kv_rows].clone()
            sd[p + "self_attn.v_proj.bias"] = w["qkv_b"][q_rows + kv_rows:].clone()
        sd[p + "self_attn.o_proj.weight"] = w["o_w"].clone()
        if "q_norm" in w:
            sd[p + "self_attn.q_norm.weight"] = w["q_norm"].clone()
            sd[p + "self_attn.k_norm.weight"] = w["k_norm"].clone()
        sd[p + "mlp.gate_proj.weight"] = w["gu_w"][0::2].clone()
        sd[p + "mlp.up_proj.weight"] = w["gu_w"][1::2].clone()
        sd[p + "mlp.down_proj.weight"] = w["down_w"].clone()
        sd[p + "input_layernorm.weight"] = w["input_norm"].clone()
        sd[p + "post_attention_layernorm.weight"] = w["post_norm"].clone()
    h = lays["head"].views(units["head"])
    sd[L + "norm.weight"] = h["final_norm"].clone()
    sd["lm_head.weight"] = h["lm_head"].clone()
    if spec.vision is not None:
        vs = spec.vision
        v = lays["visual"].views(units["visual"])
        V = "model.visual."
        sd[V + "patch_embed.proj.weight"] = v["patch_w"].reshape(vs.hidden_size, vs.in_channels, vs.temporal_patch_size,
                                                                 vs.patch_size, vs.patch_size).clone()
        if spec.vision_arch in ("qwen25", "reference"):
            for j in range(vs.depth):
                b, q = f"b{j}.", f"{V}blocks.{j}."
                sd[q + "norm1.weight"] = v[b + "n1_w"].clone()
                sd[q + "norm2.weight"] = v[b + "n2_w"].clone()
                for src in ("qkv", "proj"):
                    sd[q + f"attn.{src}.weight"] = v[b + src + "_w"].clone()
                    sd[q + f"attn.{src}.bias"] = v[b + src + "_b"].clone()
                for name, rows in (("gate_proj", slice(0, None, 2)), ("up_proj", slice(1, None, 2))):
                    sd[q + f"mlp.{name}.weight"] = v[b + "gu_w"][rows].clone()
                    sd[q + f"mlp.{name}.bias"] = v[b + "gu_b"][rows].clone()
                sd[q + "mlp.down_proj.weight"] = v[b + "down_w"].clone()
                sd[q + "mlp.down_proj.bias"] = v[b + "down_b"].clone()
            sd[V + "merger.ln_q.weight"] = v["m.norm_w"].clone()
            for src, dst in (("fc1", "mlp.0"), ("fc2", "mlp.2")):
                sd[f"{V}merger.{dst}.weight"] = v[f"m.{src}_w"].clone()
                sd[f"{V}merger.{dst}.bias"] = v[f"m.{src}_b"].clone()
            if spec.vision_arch == "reference":
                for k in range(len(vs.deepstack_visual_indexes)):
                    q = f"{V}deepstack_merger_list.{k}."
                    sd[q + "norm.weight"] = v[f"d{k}.norm_w"].clone()
                    for src, dst in (("fc1", "linear_fc1"), ("fc2", "linear_fc2")):
                        sd[q + f"{dst}.weight"] = v[f"d{k}.{src}_w"].clone()
                        sd[q + f"{dst}.bias"] = v[f"d{k}.{src}_b"].clone()
            return sd
        sd[V + "patch_embed.proj.bias"] = v["patch_b"].clone()
        if "pos_embed" in v:
            sd[V + "pos_embed.weight"] = v["pos_embed"].clone()
        for j in range(vs.depth):
            for src, dst in (("n1", "norm1"), ("n2", "norm2"), ("qkv", "attn.qkv"), ("proj", "attn.proj"),
                             ("fc1", "mlp.linear_fc1"), ("fc2", "mlp.linear_fc2")):
                sd[f"{V}blocks.{j}.{dst}.weight"] = v[f"b{j}.{src}_w"].clone()
                sd[f"{V}blocks.{j}.{dst}.bias"] = v[f"b{j}.{src}_b"].clone()
        groups = [("m.", "merger")] + [(f"d{k}.", f"deepstack_merger_list.{k}") for k in range(len(vs.deepstack_visual_indexes))]
        for src_p, dst_p in groups:
            for src, dst in (("norm", "norm"), ("fc1", "linear_fc1"), ("fc2", "linear_fc2")):
                sd[f"{V}{dst_p}.{dst}.weight"] = v[f"{src_p}{src}_w"].clone()
                sd[f"{V}{dst_p}.{dst}.bias"] = v[f"{src_p}{src}_b"].clone()
    return sd


def load_hf_config(hf_dir: str) -> Dict[str, Any]:
    with open(os.path.join(hf_dir, "config.json")) as fh:
        return json.load(fh)


def load_hf_units(hf_dir: str, spec: Optional[Qwen3VLSpec] = None, dtype=torch.float32):
    from safetensors import safe_open

    spec = spec or spec_from_config(load_hf_config(hf_dir))
    paths = sorted(glob.glob(os.path.join(hf_dir, "*.safetensors")))
    if not paths:
        raise FileNotFoundError(f"No safetensors files found in {hf_dir}")
    sd: Dict[str, torch.Tensor] = {}
    for path in paths:
        with safe_open(path, framework="pt", device="cpu") as f:
            for key in f.keys():
                sd[key] = f.get_tensor(key)
    return spec, hf_state_dict_to_units(spec, sd, dtype=dtype)


def create_model_from_hf(hf_dir: str):
    """-> (Qwen3VLModel on CPU, Flax-named fp32 NumPy params tree)."""
    from vlmrl.models.qwen3vl.api import Qwen3VLModel

    spec, units = load_hf_units(hf_dir)
    return Qwen3VLModel(spec, units=units, device="cpu", dtype=torch.float32), units_to_flax(spec, units)


def create_model_from_ckpt(ckpt_dir: str, device="cpu", dtype=torch.float32):
    """-> (Qwen3VLModel, params tree) from ``<dir>/config.json`` + ``<dir>/params.pkl``."""
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.utils.checkpoint import Checkpoint

    spec = spec_from_config(load_hf_config(ckpt_dir))
    params = Checkpoint(os.path.join(ckpt_dir, "params.pkl"), parallel=False).load_as_dict()["params"]
    units = flax_to_units(spec, params, dtype=dtype, device=device)
    return Qwen3VLModel(spec, units=units, device=device, dtype=dtype), params


__all__ = ["hf_state_dict_to_units", "units_to_hf_state_dict", "load_hf_config", "load_hf_units",
           "create_model_from_hf", "create_model_from_ckpt"]
