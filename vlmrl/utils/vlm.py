"""Image preprocessing, chat-prompt builders and logit-masking helpers.

Behavioural counterpart of reference ``utils/vlm.py:15-258``:

* ``smart_resize`` — snap (H, W) to multiples of ``patch*merge`` inside a pixel
  budget (reference ``utils/vlm.py:21-49``).
* ``preprocess_image`` — PIL bicubic resize, CLIP normalisation and the
  merge-window-ordered patch flattening that the vision tower consumes
  (reference ``utils/vlm.py:52-147``).  Rows are ``C*Tp*P*P`` wide and ordered
  (t, h-block, w-block, h-in-block, w-in-block); inside a row the order is
  (channel, temporal, py, px), which is exactly the Conv3d weight flattening.
* prompt builders / ``extract_assistant`` / ``token_positions``
  (reference ``utils/vlm.py:150-200``).
* ``apply_top_p_logits`` / ``mask_logits_topk_topp`` — the torch oracle of the
  sampler's masking (reference ``utils/vlm.py:203-258``); the GPU sampler
  kernel (``vlmrl.ops.sampling``) never materialises a masked vocab row.

The GPU patchify kernel for synthetic uint8 images is ``vlmrl.ops.patchify``.
"""

from __future__ import annotations

import math
import os
from typing import Any, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

CLIP_MEAN = np.array([0.48145466, 0.4578275, 0.40821073], dtype=np.float32)
CLIP_STD = np.array([0.26862954, 0.26130258, 0.27577711], dtype=np.float32)
DEFAULT_MIN_PIXELS = 56 * 56
DEFAULT_MAX_PIXELS = 12845056

MASK_VALUE = -1e9


def smart_resize(height: int, width: int, *, factor: int, min_pixels: int, max_pixels: int) -> Tuple[int, int]:
    """Return (h, w), both multiples of ``factor``, with ``min_pixels <= h*w <= max_pixels``."""
    if height <= 0 or width <= 0:
        raise ValueError("Image dimensions must be positive")
    lo, hi = sorted((height, width))
    if hi / lo > 200:
        raise ValueError("absolute aspect ratio must be smaller than 200")

    def snap(v: float, fn) -> int:
        return max(factor, int(fn(v / factor)) * factor)

    h, w = snap(height, round), snap(width, round)
    if h * w > max_pixels:
        scale = math.sqrt(height * width / float(max_pixels))
        h, w = snap(height / scale, math.floor), snap(width / scale, math.floor)
    elif h * w < min_pixels:
        scale = math.sqrt(float(min_pixels) / (height * width))
        h, w = snap(height * scale, math.ceil), snap(width * scale, math.ceil)
    return int(h), int(w)


def _to_pil(image: Any):
    from PIL import Image

    if isinstance(image, (str, os.PathLike)):
        path = os.fspath(image)
        if not os.path.exists(path):
            raise FileNotFoundError(f"Image file not found: {path}")
        with Image.open(path) as img:
            return img.convert("RGB")
    if hasattr(image, "convert") and hasattr(image, "size"):
        return image.convert("RGB")
    arr = np.asarray(image)
    if arr.ndim != 3 or arr.shape[2] not in (3, 4):
        raise ValueError("Unsupported image array shape; expected HWC with 3 or 4 channels")
    return Image.fromarray(arr[:, :, :3].astype(np.uint8), mode="RGB")


def patchify(frames: np.ndarray, *, patch_size: int, spatial_merge_size: int, temporal_patch_size: int) -> Tuple[np.ndarray, np.ndarray]:
    """Flatten normalised frames ``[F, C, H, W]`` into vision-tower rows.

    Frames are padded (by repeating the last one) to a multiple of the temporal
    patch.  Returns ``(rows [T*H'*W', C*Tp*P*P], grid_thw [1, 3])``.
    """
    if frames.shape[0] % temporal_patch_size:
        pad = temporal_patch_size - frames.shape[0] % temporal_patch_size
        frames = np.concatenate([frames, np.repeat(frames[-1:], pad, axis=0)], axis=0)
    f, c, h, w = frames.shape
    p, m, tp = patch_size, spatial_merge_size, temporal_patch_size
    gt, gh, gw = f // tp, h // p, w // p
    if gh == 0 or gw == 0:
        raise ValueError("Resized image too small for given patch size")
    if gh * p != h or gw * p != w:
        raise ValueError("Resized dimensions must be divisible by patch_size")
    if gh % m or gw % m:
        raise ValueError("Grid dimensions must be divisible by spatial_merge_size")
    # axes: (t, tp, c, hb, hm, py, wb, wm, px) -> (t, hb, wb, hm, wm, c, tp, py, px)
    x = frames.reshape(gt, tp, c, gh // m, m, p, gw // m, m, p)
    x = x.transpose(0, 3, 6, 4, 7, 2, 1, 5, 8)
    rows = np.ascontiguousarray(x.reshape(gt * gh * gw, c * tp * p * p))
    return rows, np.array([[gt, gh, gw]], dtype=np.int64)


def preprocess_image(
    image: Union[str, Any],
    *,
    patch_size: int,
    spatial_merge_size: int,
    temporal_patch_size: int,
    min_pixels: int = DEFAULT_MIN_PIXELS,
    max_pixels: int = DEFAULT_MAX_PIXELS,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Path / PIL image / HWC array -> (pixel rows fp32 [N, C*Tp*P*P], grid_thw int64 [1, 3])."""
    from PIL import Image

    pil = _to_pil(image)
    width, height = pil.size
    rh, rw = smart_resize(height, width, factor=patch_size * spatial_merge_size,
                          min_pixels=min_pixels, max_pixels=max_pixels)
    if (rw, rh) != (width, height):
        pil = pil.resize((rw, rh), Image.Resampling.BICUBIC)
    arr = (np.asarray(pil, dtype=np.float32) / 255.0 - CLIP_MEAN) / CLIP_STD
    frames = arr.transpose(2, 0, 1)[None]
    rows, grid = patchify(frames, patch_size=patch_size, spatial_merge_size=spatial_merge_size,
                          temporal_patch_size=temporal_patch_size)
    return torch.from_numpy(rows), torch.from_numpy(grid)


def decode_tokens(tokenizer, token_ids: Sequence[int]) -> str:
    return tokenizer.decode(list(token_ids), skip_special_tokens=True, clean_up_tokenization_spaces=False)


def _vision_block(n: int) -> str:
    return "<|vision_start|>" + "<|image_pad|>" * int(n) + "<|vision_end|>"


def chat_prompt_with_image(num_vision_tokens: int, question: str) -> str:
    return chat_prompt_with_images([num_vision_tokens], question)


def chat_prompt_with_images(num_tokens_list: Sequence[int], question: str) -> str:
    blocks = "".join(_vision_block(n) for n in num_tokens_list)
    return f"<|im_start|>user\n{blocks}{question}<|im_end|>\n<|im_start|>assistant\n"


def extract_assistant(full_text: str) -> Optional[str]:
    head, tail = "<|im_start|>assistant\n", "<|im_end|>"
    pos = full_text.rfind(head)
    if pos < 0:
        return None
    body = full_text[pos + len(head):]
    end = body.find(tail)
    return body if end < 0 else body[:end]


def token_positions(tokens: torch.Tensor, pad_id: int) -> Tuple[torch.Tensor, torch.Tensor]:
    mask = (tokens != pad_id).to(torch.int32)
    pos = torch.cumsum(mask, dim=-1) - 1
    return torch.where(mask > 0, pos, torch.zeros_like(pos)), mask


def apply_top_p_logits(logits: torch.Tensor, top_p: Optional[float]) -> torch.Tensor:
    """Exact nucleus filter over the full vocab (O(V log V) oracle)."""
    if top_p is None or not (0.0 < float(top_p) < 1.0):
        return logits
    vals, order = torch.sort(logits.float(), dim=-1, descending=True)
    cum = torch.cumsum(torch.softmax(vals, dim=-1), dim=-1)
    keep = cum <= float(top_p)
    keep[..., 0] = True
    vals = torch.where(keep, vals, torch.full_like(vals, MASK_VALUE))
    out = torch.full_like(vals, MASK_VALUE)
    return out.scatter(-1, order, vals)


def mask_logits_topk_topp(logits: torch.Tensor, *, top_k: Optional[int], top_p: Optional[float]) -> torch.Tensor:
    """Top-k shortlist, then nucleus inside the shortlist; everything else -> -1e9."""
    use_k = top_k is not None and int(top_k) > 0
    use_p = top_p is not None and 0.0 < float(top_p) < 1.0
    if not use_k:
        return apply_top_p_logits(logits, top_p) if use_p else logits
    k = min(int(top_k), logits.shape[-1])
    vals, idx = torch.topk(logits.float(), k, dim=-1)
    if use_p:
        cum = torch.cumsum(torch.softmax(vals, dim=-1), dim=-1)
        keep = cum <= float(top_p)
        keep[..., 0] = True
        vals = torch.where(keep, vals, torch.full_like(vals, MASK_VALUE))
    out = torch.full(logits.shape, MASK_VALUE, dtype=torch.float32, device=logits.device)
    return out.scatter(-1, idx, vals)


__all__ = [
    "CLIP_MEAN", "CLIP_STD", "DEFAULT_MIN_PIXELS", "DEFAULT_MAX_PIXELS", "MASK_VALUE",
    "smart_resize", "patchify", "preprocess_image", "decode_tokens", "chat_prompt_with_image",
    "chat_prompt_with_images", "extract_assistant", "token_positions", "apply_top_p_logits",
    "mask_logits_topk_topp",
]
