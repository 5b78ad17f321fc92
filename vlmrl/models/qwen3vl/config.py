"""Qwen3-VL specification objects, HF-config parsing and named presets.

``spec_from_config`` reads an HF ``config.json`` dict the way reference
``models/qwen3vl/model.py:892-983`` does (``text_config`` / ``vision_config``
sections, ``rope_scaling.mrope_section`` validated against ``head_dim//2``,
``fullatt_block_indexes`` defaulting to the deepstack indexes) and additionally
keeps the fields an HF-faithful model needs (``num_position_embeddings``,
``tie_word_embeddings``, special token ids, ``hidden_act``).

Presets:

* ``tiny``   — the CPU/gloo test model (ViT 2x64, decoder 2x128, vocab 1024).
* ``qwen3vl_4b`` — Qwen3-VL-4B architecture (ViT 24x1024 -> 2560, decoder
  36x2560, 32q/8kv heads of 128, SwiGLU 9728, vocab 151936, tied embeddings).
* ``qwen3vl_8b`` — decoder 36x4096, SwiGLU 12288, untied lm_head, same ViT with
  output width 4096.
"""

from __future__ import annotations

import copy
from dataclasses import asdict, dataclass, field, replace
from typing import Any, Dict, Optional, Sequence, Tuple

IMAGE_TOKEN_ID = 151655
VIDEO_TOKEN_ID = 151656
VISION_START_TOKEN_ID = 151652
VISION_END_TOKEN_ID = 151653


@dataclass
class TextBackboneSpec:
    hidden_size: int
    num_attention_heads: int
    num_hidden_layers: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    rope_theta: float
    rope_section: Sequence[int]
    rope_scaling_type: Optional[str] = None
    rope_scaling_factor: Optional[float] = None
    mrope_interleaved: bool = True
    rms_norm_eps: float = 1e-6
    vocab_size: int = 151936
    tie_word_embeddings: bool = True
    attention_bias: bool = False
    # per-head RMSNorm on q and k before RoPE (Qwen3); Qwen2.5 rotates the raw projections
    qk_norm: bool = True


@dataclass
class VisionBackboneSpec:
    hidden_size: int
    out_hidden_size: int
    depth: int
    num_heads: int
    intermediate_size: int
    patch_size: int
    temporal_patch_size: int
    spatial_merge_size: int
    window_size: int = 0
    in_channels: int = 3
    fullatt_block_indexes: Sequence[int] = ()
    num_position_embeddings: Optional[int] = 2304
    deepstack_visual_indexes: Sequence[int] = ()
    hidden_act: str = "gelu_pytorch_tanh"
    tokens_per_second: float = 2.0

    @property
    def patch_volume(self) -> int:
        return self.in_channels * self.temporal_patch_size * self.patch_size * self.patch_size

    @property
    def merged_hidden_size(self) -> int:
        return self.hidden_size * self.spatial_merge_size ** 2


@dataclass
class Qwen3VLSpec:
    text: TextBackboneSpec
    vision: Optional[VisionBackboneSpec]
    pad_token_id: Optional[int] = None
    bos_token_id: Optional[int] = None
    eos_token_id: Optional[int] = None
    image_token_id: int = IMAGE_TOKEN_ID
    video_token_id: int = VIDEO_TOKEN_ID
    vision_start_token_id: int = VISION_START_TOKEN_ID
    vision_end_token_id: int = VISION_END_TOKEN_ID
    # "hf": LayerNorm + GELU MLP ViT with learned pos-embed and full attention (HF Qwen3-VL);
    # "qwen25": RMSNorm + SwiGLU ViT with window attention and full attention at fullatt_block_indexes
    # (HF Qwen2.5-VL);
    # "reference": the Qwen3-VL tower as the reference computes it (reference models/qwen3vl/vision.py:
    # RMSNorm + biased SwiGLU blocks, no position table, windows of window_size px with full attention at
    # fullatt_block_indexes, its own rotary frequencies, RMSNorm mergers with tanh-GELU, deepstack
    # mergers), for numerical parity with parameter trees that the reference trained or converted.
    vision_arch: str = "hf"

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


def _int_list(x) -> Tuple[int, ...]:
    return tuple(int(v) for v in (x or ()))


def spec_from_config(cfg: Dict[str, Any]) -> Qwen3VLSpec:
    text_cfg = cfg.get("text_config", cfg)
    rope_cfg = text_cfg.get("rope_scaling") or text_cfg.get("rope_parameters") or cfg.get("rope_scaling") or {}
    head_dim = int(text_cfg.get("head_dim") or text_cfg["hidden_size"] // text_cfg["num_attention_heads"])
    vision_cfg = cfg.get("vision_config")

    scaling_type = rope_cfg.get("type", rope_cfg.get("rope_type")) if isinstance(rope_cfg, dict) else None
    if scaling_type in ("default", "mrope"):
        scaling_type = None
    qwen25 = str(cfg.get("model_type", "")).startswith("qwen2_5_vl") or str(cfg.get("model_type", "")) == "qwen2_vl"
    scaling_factor = rope_cfg.get("factor", rope_cfg.get("finetuned_factor")) if isinstance(rope_cfg, dict) else None
    interleaved = bool(rope_cfg.get("mrope_interleaved", False)) if isinstance(rope_cfg, dict) else False
    section = rope_cfg.get("mrope_section") if isinstance(rope_cfg, dict) else None
    if section is None:
        if vision_cfg is not None:
            raise ValueError("Missing rope_scaling.mrope_section for vision model; expected 3-tuple summing to head_dim//2.")
        section = [head_dim // 2]
    section = [int(s) for s in section]
    if vision_cfg is not None and len(section) != 3:
        raise ValueError("rope_scaling.mrope_section must have 3 entries (t,h,w) for vision models")
    if not interleaved and sum(section) != head_dim // 2:
        raise ValueError(f"Sum of rope_scaling.mrope_section must equal head_dim//2 ({head_dim // 2}); got {sum(section)}")
    theta = text_cfg.get("rope_theta", (rope_cfg or {}).get("rope_theta", cfg.get("rope_theta", 10000.0)))

    text = TextBackboneSpec(
        hidden_size=int(text_cfg["hidden_size"]), num_attention_heads=int(text_cfg["num_attention_heads"]),
        num_hidden_layers=int(text_cfg["num_hidden_layers"]), num_key_value_heads=int(text_cfg["num_key_value_heads"]),
        head_dim=head_dim, intermediate_size=int(text_cfg["intermediate_size"]), rope_theta=float(theta),
        rope_section=tuple(section), rope_scaling_type=scaling_type,
        rope_scaling_factor=float(scaling_factor) if scaling_factor is not None else None,
        mrope_interleaved=interleaved, rms_norm_eps=float(text_cfg.get("rms_norm_eps", 1e-6)),
        vocab_size=int(text_cfg["vocab_size"]),
        tie_word_embeddings=bool(cfg.get("tie_word_embeddings", text_cfg.get("tie_word_embeddings", False))),
        attention_bias=bool(text_cfg.get("attention_bias", qwen25)),
        qk_norm=not qwen25,
    )
    vision = None
    if vision_cfg is not None:
        patch = int(vision_cfg.get("patch_size", vision_cfg.get("spatial_patch_size")))
        merge = int(vision_cfg.get("spatial_merge_size", 1))
        deep = _int_list(vision_cfg.get("deepstack_visual_indexes", ()))
        vision = VisionBackboneSpec(
            hidden_size=int(vision_cfg["hidden_size"]), out_hidden_size=int(vision_cfg["out_hidden_size"]),
            depth=int(vision_cfg["depth"]), num_heads=int(vision_cfg["num_heads"]),
            intermediate_size=int(vision_cfg["intermediate_size"]), patch_size=patch,
            temporal_patch_size=int(vision_cfg.get("temporal_patch_size", vision_cfg.get("temporal_patch", 1))),
            spatial_merge_size=merge, window_size=int(vision_cfg.get("window_size", patch * merge)),
            in_channels=int(vision_cfg.get("in_channels", vision_cfg.get("in_chans", 3))),
            fullatt_block_indexes=_int_list(vision_cfg.get("fullatt_block_indexes", deep)),
            num_position_embeddings=vision_cfg.get("num_position_embeddings"),
            deepstack_visual_indexes=deep, hidden_act=str(vision_cfg.get("hidden_act", "gelu_pytorch_tanh")),
            tokens_per_second=float(vision_cfg.get("tokens_per_second", 2.0)),
        )
    return Qwen3VLSpec(
        text=text, vision=vision, pad_token_id=cfg.get("pad_token_id"), bos_token_id=cfg.get("bos_token_id"),
        eos_token_id=cfg.get("eos_token_id"), image_token_id=int(cfg.get("image_token_id", IMAGE_TOKEN_ID)),
        video_token_id=int(cfg.get("video_token_id", VIDEO_TOKEN_ID)),
        vision_start_token_id=int(cfg.get("vision_start_token_id", VISION_START_TOKEN_ID)),
        vision_end_token_id=int(cfg.get("vision_end_token_id", VISION_END_TOKEN_ID)),
        vision_arch="qwen25" if qwen25 else str(cfg.get("vision_arch", "hf")),
    )


def spec_to_config(spec: Qwen3VLSpec) -> Dict[str, Any]:
    """Inverse of ``spec_from_config``: an HF-style ``config.json`` dict."""
    t = spec.text
    qwen25 = spec.vision_arch == "qwen25"
    cfg: Dict[str, Any] = {
        "model_type": "qwen2_5_vl" if qwen25 else "qwen3_vl",
        "architectures": ["Qwen2_5_VLForConditionalGeneration" if qwen25 else "Qwen3VLForConditionalGeneration"],
        "tie_word_embeddings": t.tie_word_embeddings,
        "image_token_id": spec.image_token_id, "video_token_id": spec.video_token_id,
        "vision_start_token_id": spec.vision_start_token_id, "vision_end_token_id": spec.vision_end_token_id,
        "text_config": {
            "hidden_size": t.hidden_size, "num_attention_heads": t.num_attention_heads,
            "num_hidden_layers": t.num_hidden_layers, "num_key_value_heads": t.num_key_value_heads,
            "head_dim": t.head_dim, "intermediate_size": t.intermediate_size, "rope_theta": t.rope_theta,
            "rms_norm_eps": t.rms_norm_eps, "vocab_size": t.vocab_size, "attention_bias": t.attention_bias,
            "hidden_act": "silu", "tie_word_embeddings": t.tie_word_embeddings,
            "rope_scaling": {"rope_type": t.rope_scaling_type or "default", "mrope_section": list(t.rope_section),
                             "mrope_interleaved": t.mrope_interleaved},
        },
    }
    for k in ("pad_token_id", "bos_token_id", "eos_token_id"):
        if getattr(spec, k) is not None:
            cfg[k] = getattr(spec, k)
    if spec.vision is not None:
        v = spec.vision
        cfg["vision_config"] = {
            "hidden_size": v.hidden_size, "out_hidden_size": v.out_hidden_size, "depth": v.depth,
            "num_heads": v.num_heads, "intermediate_size": v.intermediate_size, "patch_size": v.patch_size,
            "temporal_patch_size": v.temporal_patch_size, "spatial_merge_size": v.spatial_merge_size,
            "in_channels": v.in_channels, "num_position_embeddings": v.num_position_embeddings,
            "deepstack_visual_indexes": list(v.deepstack_visual_indexes), "hidden_act": v.hidden_act,
        }
        if qwen25:
            cfg["vision_config"].update(window_size=v.window_size, fullatt_block_indexes=list(v.fullatt_block_indexes),
                                        tokens_per_second=int(v.tokens_per_second) if float(v.tokens_per_second).is_integer()
                                        else v.tokens_per_second, in_chans=v.in_channels)
            cfg["vision_config"].pop("num_position_embeddings")
            cfg["vision_config"].pop("deepstack_visual_indexes")
            cfg["text_config"]["rope_scaling"] = {"type": "mrope", "mrope_section": list(t.rope_section)}
        elif spec.vision_arch == "reference":
            cfg["vision_arch"] = "reference"
            cfg["vision_config"].update(window_size=v.window_size, fullatt_block_indexes=list(v.fullatt_block_indexes))
    return cfg


def _vision_4b(out_hidden: int) -> VisionBackboneSpec:
    return VisionBackboneSpec(hidden_size=1024, out_hidden_size=out_hidden, depth=24, num_heads=16,
                              intermediate_size=4096, patch_size=16, temporal_patch_size=2, spatial_merge_size=2,
                              num_position_embeddings=2304, deepstack_visual_indexes=(5, 11, 17),
                              fullatt_block_indexes=(5, 11, 17))


def _qwen25_vision(out_hidden: int, depth: int = 32) -> VisionBackboneSpec:
    return VisionBackboneSpec(hidden_size=1280, out_hidden_size=out_hidden, depth=depth, num_heads=16,
                              intermediate_size=3420, patch_size=14, temporal_patch_size=2, spatial_merge_size=2,
                              window_size=112, fullatt_block_indexes=(7, 15, 23, 31), num_position_embeddings=None,
                              deepstack_visual_indexes=(), hidden_act="silu", tokens_per_second=2.0)


PRESETS: Dict[str, Qwen3VLSpec] = {
    "tiny": Qwen3VLSpec(
        text=TextBackboneSpec(hidden_size=128, num_attention_heads=4, num_hidden_layers=2, num_key_value_heads=2,
                              head_dim=32, intermediate_size=384, rope_theta=5e6, rope_section=(6, 5, 5),
                              mrope_interleaved=True, vocab_size=1024, tie_word_embeddings=True),
        vision=VisionBackboneSpec(hidden_size=64, out_hidden_size=128, depth=2, num_heads=4, intermediate_size=256,
                                  patch_size=16, temporal_patch_size=2, spatial_merge_size=2,
                                  num_position_embeddings=256, deepstack_visual_indexes=(1,),
                                  fullatt_block_indexes=(1,)),
        image_token_id=1024 - 2, video_token_id=1024 - 1, vision_start_token_id=1024 - 4,
        vision_end_token_id=1024 - 3, eos_token_id=1024 - 5, pad_token_id=1024 - 7,
    ),
    "qwen3vl_4b": Qwen3VLSpec(
        text=TextBackboneSpec(hidden_size=2560, num_attention_heads=32, num_hidden_layers=36, num_key_value_heads=8,
                              head_dim=128, intermediate_size=9728, rope_theta=5e6, rope_section=(24, 20, 20),
                              mrope_interleaved=True, vocab_size=151936, tie_word_embeddings=True),
        vision=_vision_4b(2560), eos_token_id=151645, pad_token_id=151643,
    ),
    "qwen3vl_8b": Qwen3VLSpec(
        text=TextBackboneSpec(hidden_size=4096, num_attention_heads=32, num_hidden_layers=36, num_key_value_heads=8,
                              head_dim=128, intermediate_size=12288, rope_theta=5e6, rope_section=(24, 20, 20),
                              mrope_interleaved=True, vocab_size=151936, tie_word_embeddings=False),
        vision=_vision_4b(4096), eos_token_id=151645, pad_token_id=151643,
    ),
    "tiny_qwen25": Qwen3VLSpec(
        text=TextBackboneSpec(hidden_size=128, num_attention_heads=4, num_hidden_layers=2, num_key_value_heads=2,
                              head_dim=32, intermediate_size=384, rope_theta=1e6, rope_section=(4, 6, 6),
                              mrope_interleaved=False, vocab_size=1024, tie_word_embeddings=True,
                              attention_bias=True, qk_norm=False),
        vision=VisionBackboneSpec(hidden_size=64, out_hidden_size=128, depth=3, num_heads=4, intermediate_size=160,
                                  patch_size=14, temporal_patch_size=2, spatial_merge_size=2, window_size=56,
                                  fullatt_block_indexes=(1,), num_position_embeddings=None, hidden_act="silu"),
        image_token_id=1024 - 2, video_token_id=1024 - 1, vision_start_token_id=1024 - 4,
        vision_end_token_id=1024 - 3, eos_token_id=1024 - 5, pad_token_id=1024 - 7, vision_arch="qwen25",
    ),
    "qwen25vl_3b": Qwen3VLSpec(
        text=TextBackboneSpec(hidden_size=2048, num_attention_heads=16, num_hidden_layers=36, num_key_value_heads=2,
                              head_dim=128, intermediate_size=11008, rope_theta=1e6, rope_section=(16, 24, 24),
                              mrope_interleaved=False, vocab_size=151936, tie_word_embeddings=True,
                              attention_bias=True, qk_norm=False),
        vision=_qwen25_vision(2048), eos_token_id=151645, pad_token_id=151643, vision_arch="qwen25",
    ),
    "qwen25vl_7b": Qwen3VLSpec(
        text=TextBackboneSpec(hidden_size=3584, num_attention_heads=28, num_hidden_layers=28, num_key_value_heads=4,
                              head_dim=128, intermediate_size=18944, rope_theta=1e6, rope_section=(16, 24, 24),
                              mrope_interleaved=False, vocab_size=152064, tie_word_embeddings=False,
                              attention_bias=True, qk_norm=False),
        vision=_qwen25_vision(3584), eos_token_id=151645, pad_token_id=151643, vision_arch="qwen25",
    ),
}


def get_preset(name: str, **overrides) -> Qwen3VLSpec:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")
    spec = copy.deepcopy(PRESETS[name])
    return replace(spec, **overrides) if overrides else spec


def tiny_token_ids(spec: Qwen3VLSpec) -> Dict[str, int]:
    """Special-token ids of a spec (the tiny preset keeps them inside its 1024-entry vocab)."""
    return {"<|image_pad|>": spec.image_token_id, "<|video_pad|>": spec.video_token_id,
            "<|vision_start|>": spec.vision_start_token_id, "<|vision_end|>": spec.vision_end_token_id,
            "<|im_end|>": spec.eos_token_id if spec.eos_token_id is not None else 0,
            "<|endoftext|>": spec.pad_token_id if spec.pad_token_id is not None else 0}


__all__ = ["TextBackboneSpec", "VisionBackboneSpec", "Qwen3VLSpec", "spec_from_config", "spec_to_config",
           "PRESETS", "get_preset", "tiny_token_ids", "IMAGE_TOKEN_ID", "VIDEO_TOKEN_ID",
           "VISION_START_TOKEN_ID", "VISION_END_TOKEN_ID"]
