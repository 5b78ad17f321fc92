"""Qwen3-VL: config/spec, parameter layout, executor, weights conversion (reference ``models/qwen3vl/__init__.py``)."""

from vlmrl.models.qwen3vl.config import (PRESETS, Qwen3VLSpec, TextBackboneSpec, VisionBackboneSpec, get_preset,
                                         spec_from_config, spec_to_config)
from vlmrl.models.qwen3vl.model import KVCache, LocalParams, PackedBatch, TextDecoder, VisionEmbeddings
from vlmrl.models.qwen3vl.rope import get_rope_index, mrope_cos_sin
from vlmrl.models.qwen3vl.api import Qwen3VLModel
from vlmrl.models.qwen3vl.weights import create_model_from_ckpt, create_model_from_hf

__all__ = ["Qwen3VLModel", "Qwen3VLSpec", "TextBackboneSpec", "VisionBackboneSpec", "PRESETS", "get_preset",
           "spec_from_config", "spec_to_config", "KVCache", "LocalParams", "PackedBatch", "TextDecoder",
           "VisionEmbeddings", "get_rope_index", "mrope_cos_sin", "create_model_from_ckpt", "create_model_from_hf"]
