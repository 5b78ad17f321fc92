"""Qwen2.5-VL model family (reference ``models/qwen25vl/{model,vision}.py``).

Qwen2.5-VL runs on the same executor as Qwen3-VL (``vlmrl.models.qwen3vl``):
the spec selects the differences, so every kernel, the sampler, the trainer
and FSDP work unchanged.

* text: q/k/v projections with bias and no q/k RMSNorm (``qk_norm=False``:
  the RoPE kernels rotate the raw projections); chunked MRoPE sections
  ``[16, 24, 24]`` (``mrope_interleaved=False``); ``rope_theta`` 1e6;
* vision (``vision_arch="qwen25"``): RMSNorm blocks with a biased SwiGLU MLP,
  window attention of ``window_size`` (112) pixels with full attention at
  ``fullatt_block_indexes``, no deepstack, one RMSNorm merger;
* positions: ``get_rope_index`` scales a video's frame index by seconds per
  grid x ``tokens_per_second`` (reference ``models/qwen25vl/model.py:159-333``).

``create_model_from_hf`` / ``create_model_from_ckpt`` read the HF config's
``model_type`` (``qwen2_5_vl``) and build the matching spec.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import numpy as np

from vlmrl.models.qwen3vl.api import Qwen3VLModel as Qwen25VLModel
from vlmrl.models.qwen3vl.config import PRESETS as _ALL_PRESETS
from vlmrl.models.qwen3vl.config import Qwen3VLSpec as Qwen25VLSpec
from vlmrl.models.qwen3vl.config import get_preset, spec_from_config, spec_to_config
from vlmrl.models.qwen3vl.rope import get_rope_index as _rope_index
from vlmrl.models.qwen3vl.weights import (create_model_from_ckpt, create_model_from_hf, hf_state_dict_to_units,
                                          units_to_hf_state_dict)

VIDEO_TOKEN_ID = 151656
PRESETS = {k: v for k, v in _ALL_PRESETS.items() if v.vision_arch == "qwen25"}


def get_rope_index(token_ids, image_grids: Sequence[Tuple[int, int, int]], *, spatial_merge_size: int,
                   image_token_id: int, video_token_id: Optional[int] = None,
                   video_grids: Sequence[Tuple[int, int, int]] = (), second_per_grid_ts: Sequence[float] = (),
                   tokens_per_second: float = 2.0) -> Tuple[np.ndarray, int]:
    """Qwen2.5-VL 3-axis positions for one sequence with images and videos in order of appearance.

    Image frames all take temporal index 0; video grid g advances
    ``int(frame * second_per_grid_ts[g] * tokens_per_second)`` per frame.
    """
    ids = np.asarray(token_ids, dtype=np.int64).reshape(-1)
    vid = int(video_token_id) if video_token_id is not None else VIDEO_TOKEN_ID
    grids, scales = [], []
    ii = vi = 0
    i = 0
    n = len(ids)
    while i < n:
        if ids[i] == image_token_id or ids[i] == vid:
            is_video = ids[i] == vid
            j = i
            while j < n and ids[j] == ids[i]:
                j += 1
            if is_video:
                grids.append(tuple(video_grids[vi]))
                sec = float(second_per_grid_ts[vi]) if vi < len(second_per_grid_ts) else 1.0
                scales.append(sec * float(tokens_per_second))
                vi += 1
            else:
                grids.append(tuple(image_grids[ii]))
                scales.append(0.0)
                ii += 1
            i = j
        else:
            i += 1
    return _rope_index(ids, grids, spatial_merge_size=spatial_merge_size, image_token_id=image_token_id,
                       video_token_id=vid, t_scale=scales)


__all__ = ["Qwen25VLModel", "Qwen25VLSpec", "PRESETS", "get_preset", "spec_from_config", "spec_to_config",
           "get_rope_index", "create_model_from_hf", "create_model_from_ckpt", "hf_state_dict_to_units",
           "units_to_hf_state_dict", "VIDEO_TOKEN_ID"]
