"""Keyword-coverage captioning demo env (reference ``envs/vision_caption.py:24-121``).

Fifteen fixed (question, image, keywords) prompts over a folder of demo images;
reward = fraction of keywords present (case-insensitive) in the response.  The
package ships drawn versions of the seven scenes (``vlmrl/assets/imgs``, made by
``vlmrl.assets.make_demo_images``); with another ``asset_root`` whose files are
missing, the env substitutes a deterministic random image so that it still runs.
"""

from __future__ import annotations

import os
import zlib
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence, Tuple

import numpy as np

from vlmrl.envs.base import BaseEnv, BaseState, resolve_eos_id
from vlmrl.utils.vlm import decode_tokens

CAPTION_TASKS: Tuple[Tuple[str, str, Tuple[str, ...]], ...] = (
    ("Describe the news content shown in the image.", "foxnews.png", ("news", "fox", "futures")),
    ("Give a concise description of the diagram.", "foxnews.png", ("nasdaq", "futures", "trading")),
    ("Explain what the Nasdaq futures are trading at in the image.", "foxnews.png", ("nasdaq", "futures", "trading")),
    ("Describe what is happening in this image.", "f35_takeoff.png", ("aircraft", "jet", "takeoff", "military")),
    ("What type of aircraft is shown in this image?", "f35_takeoff.png", ("f-35", "fighter", "jet", "aircraft")),
    ("Describe the ceremony shown in the image.", "japanese_ceremony.png", ("ceremony", "traditional", "wedding", "japanese")),
    ("What cultural event is taking place in this image?", "japanese_ceremony.png", ("ceremony", "traditional", "cultural", "ritual")),
    ("Describe the landscape in this image.", "mountain_landscape.png", ("mountain", "landscape", "nature", "scenic")),
    ("What natural features are visible in this image?", "mountain_landscape.png", ("mountain", "peak", "terrain", "wilderness")),
    ("Describe what the animal is doing in this image.", "panda_climbing.png", ("panda", "climbing", "bear", "animal")),
    ("What type of animal is shown in the image?", "panda_climbing.png", ("panda", "bear", "endangered", "wildlife")),
    ("Describe the aerial view in this image.", "stadium_aerial.png", ("stadium", "aerial", "sports", "venue")),
    ("What structure is visible from above in this image?", "stadium_aerial.png", ("stadium", "arena", "building", "architecture")),
    ("Describe the workspace setup in this image.", "coffee_laptop.png", ("laptop", "coffee", "workspace", "desk")),
    ("What items are visible on the desk in this image?", "coffee_laptop.png", ("laptop", "computer", "coffee", "work")),
)


@dataclass(frozen=True)
class VisionCaptionSample:
    question: str
    image_path: str
    keywords: Tuple[str, ...]


@dataclass(frozen=True)
class VisionPrompt:
    question: str
    image_path: str
    keywords: Tuple[str, ...]
    image: Optional[object] = None


@dataclass(frozen=True)
class VisionCaptionState(BaseState):
    dataset_idx: int
    sample: VisionCaptionSample

    def render(self) -> str:
        return self.sample.question


def placeholder_image(name: str, size: int = 224) -> np.ndarray:
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    return rng.integers(0, 256, size=(size, size, 3), dtype=np.uint8)


class VisionCaptionEnv(BaseEnv):
    def __init__(self, tokenizer, asset_root: Optional[str] = None):
        super().__init__()
        self.tokenizer = tokenizer
        self.tokens_per_action = 128
        root = Path(asset_root) if asset_root else Path(__file__).resolve().parents[1] / "assets" / "imgs"
        self.dataset = [VisionCaptionSample(q, str(root / img), kw) for q, img, kw in CAPTION_TASKS]
        self.num_tasks = len(self.dataset)
        self.eos_token_id = resolve_eos_id(tokenizer)

    def reset(self, idx: int):
        i = idx % len(self.dataset)
        s = self.dataset[i]
        image = None if os.path.exists(s.image_path) else placeholder_image(os.path.basename(s.image_path))
        return VisionCaptionState(i, s), VisionPrompt(s.question, s.image_path, s.keywords, image)

    def step(self, state: VisionCaptionState, action_tokens: Sequence[int]):
        if self.eos_token_id is not None:
            action_tokens = self.clean_action(action_tokens, self.eos_token_id)
        text = decode_tokens(self.tokenizer, action_tokens)
        low = text.lower()
        hits = sum(1 for kw in state.sample.keywords if kw.lower() in low)
        return state, [], hits / max(len(state.sample.keywords), 1), True, {
            "response": text, "hits": hits, "num_keywords": len(state.sample.keywords),
            "keywords": list(state.sample.keywords), "question": state.sample.question,
        }


__all__ = ["VisionCaptionSample", "VisionPrompt", "VisionCaptionState", "VisionCaptionEnv", "CAPTION_TASKS"]
