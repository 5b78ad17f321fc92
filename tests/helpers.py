"""Shared builders for tests: tiny model, synthetic episodes."""

import numpy as np
import torch

from vlmrl.core.batching import pack_sequences
from vlmrl.models.qwen3vl.api import Qwen3VLModel
from vlmrl.models.qwen3vl.config import get_preset
from vlmrl.models.qwen3vl.params import init_params
from vlmrl.utils.vlm import preprocess_image


def tiny_model(seed=1, dtype=torch.float32, device="cpu"):
    spec = get_preset("tiny")
    units = init_params(spec, seed=seed)
    return spec, units, Qwen3VLModel(spec, units=units, dtype=dtype, device=device)


def tiny_episodes(spec, model, n=3, prompt_text=10, action=6, seed=0, device="cpu"):
    rng = np.random.default_rng(seed)
    seqs, plens, grids, pix, grid_list = [], [], [], [], []
    for i in range(n):
        img = rng.integers(0, 256, (64, 64, 3), dtype=np.uint8)
        p, g = preprocess_image(img, patch_size=16, spatial_merge_size=2, temporal_patch_size=2)
        pix.append(p)
        grid_list.append(tuple(g[0].tolist()))
        prompt = [spec.vision_start_token_id] + [spec.image_token_id] * 4 + [spec.vision_end_token_id]
        prompt += list(rng.integers(0, 900, prompt_text - i))
        act = list(rng.integers(0, 900, action + i))
        seqs.append(np.asarray(prompt + act))
        plens.append(len(prompt))
        grids.append([grid_list[-1]])
    vis = model.encode_vision(torch.cat(pix).to(device), grid_list)
    batch, counts = pack_sequences(spec, seqs, plens, grids, vis, device=device)
    return batch, counts, seqs, plens
