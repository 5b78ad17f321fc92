"""Offline synthetic environments for the benchmark workloads.

None of these has a counterpart in the reference: they replace dataset
downloads with deterministic, seed-derived samples of the documented shapes.

* ``SyntheticGeoEnv`` — one uniform-random RGB image per prompt, uniform-random
  prompt token ids, ground truth drawn uniformly on the sphere; reward is the
  geospot geodesic kernel on coordinates parsed from the response (the
  coordinates-only ``RewardConfig``), 0 when the response does not parse.
* ``SyntheticTrueFalseEnv`` — two images per prompt, Bernoulli(0.5) label;
  reward 1 when the first generated token id equals the fixed id for the label.
* ``SyntheticParityEnv`` — reward 1 when the first generated token id is even.

Samples are generated lazily per dataset index from ``(seed, index)`` and
cached, so repeated resets of the same index return identical uint8 arrays.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from vlmrl.envs.base import BaseEnv, BaseState, resolve_eos_id
from vlmrl.envs.geospot import COORDS_ONLY, Coords, RewardConfig, compute_reward, parse_response
from vlmrl.utils.vlm import decode_tokens


@dataclass(frozen=True)
class SyntheticPrompt:
    """Observation: raw uint8 images (HWC) and already-tokenised prompt ids."""
    images: Tuple[np.ndarray, ...]
    prompt_ids: np.ndarray
    question: Optional[str] = None
    info: Dict[str, object] = field(default_factory=dict)


@dataclass(frozen=True)
class SyntheticState(BaseState):
    idx: int
    target: object

    def render(self) -> str:
        return f"synthetic task {self.idx}"


def _rng(seed: int, idx: int) -> np.random.Generator:
    return np.random.default_rng([int(seed) & 0xFFFFFFFF, int(idx) & 0xFFFFFFFF])


class _SyntheticBase(BaseEnv):
    num_images = 1

    def __init__(self, tokenizer, *, image_size: int = 448, prompt_tokens: int = 64, num_tasks: int = 1024,
                 seed: int = 0, vocab_low: int = 0, vocab_high: Optional[int] = None, cache: bool = True):
        super().__init__()
        self.tokenizer = tokenizer
        self.eos_token_id = resolve_eos_id(tokenizer)
        self.image_size = int(image_size)
        self.prompt_tokens = int(prompt_tokens)
        self.num_tasks = int(num_tasks)
        self.seed = int(seed)
        vocab = int(getattr(tokenizer, "vocab_size", 151936))
        # random prompt ids avoid the special-token block at the top of the vocab
        self.vocab_low = int(vocab_low)
        self.vocab_high = int(vocab_high) if vocab_high is not None else min(vocab, 151643)
        self._cache: Dict[int, Tuple[SyntheticPrompt, object]] = {} if cache else None

    def _target(self, rng: np.random.Generator):
        raise NotImplementedError

    def _make(self, idx: int) -> Tuple[SyntheticPrompt, object]:
        rng = _rng(self.seed, idx)
        imgs = tuple(rng.integers(0, 256, size=(self.image_size, self.image_size, 3), dtype=np.uint8)
                     for _ in range(self.num_images))
        ids = rng.integers(self.vocab_low, self.vocab_high, size=(self.prompt_tokens,), dtype=np.int64).astype(np.int32)
        target = self._target(rng)
        return SyntheticPrompt(images=imgs, prompt_ids=ids), target

    def reset(self, idx: int):
        key = idx % self.num_tasks if self.num_tasks > 0 else idx
        if self._cache is not None and key in self._cache:
            obs, target = self._cache[key]
        else:
            obs, target = self._make(key)
            if self._cache is not None:
                self._cache[key] = (obs, target)
        return SyntheticState(idx=key, target=target), obs


def sphere_point(rng: np.random.Generator) -> Coords:
    """Uniform point on the sphere: lat = asin(2u-1), lon uniform."""
    u, v = rng.random(), rng.random()
    lat = math.degrees(math.asin(2.0 * u - 1.0))
    lon = 360.0 * v - 180.0
    return Coords(lat=max(-90.0, min(90.0, lat)), lon=max(-180.0, min(180.0, lon)))


class SyntheticGeoEnv(_SyntheticBase):
    def __init__(self, tokenizer, reward_config: RewardConfig = COORDS_ONLY, **kw):
        super().__init__(tokenizer, **kw)
        self.tokens_per_action = 128
        self.reward_config = reward_config

    def _target(self, rng):
        return sphere_point(rng)

    def step(self, state: SyntheticState, action_tokens: Sequence[int]):
        if self.eos_token_id is not None:
            action_tokens = self.clean_action(action_tokens, self.eos_token_id)
        text = decode_tokens(self.tokenizer, action_tokens).strip()
        parsed = parse_response(text)
        from vlmrl.envs.geospot import Location

        truth = Location(city="", region="", country="", coords=state.target)
        res = compute_reward(truth, parsed, self.reward_config, lambda q: None)
        d = res.d_coords
        return state, [], float(res.reward), True, {
            "final_reward": float(res.reward), "format_ok": float(parsed.format_valid),
            "has_coords": float(parsed.coords is not None),
            "coords_within_tolerance": float(res.within_tolerance),
            **({"distance_km": d} if d is not None else {}),
        }


class SyntheticTrueFalseEnv(_SyntheticBase):
    num_images = 2

    def __init__(self, tokenizer, true_id: Optional[int] = None, false_id: Optional[int] = None, **kw):
        kw.setdefault("image_size", 384)
        kw.setdefault("prompt_tokens", 48)
        super().__init__(tokenizer, **kw)
        self.tokens_per_action = 8
        enc = getattr(tokenizer, "encode", None)
        self.true_id = int(true_id) if true_id is not None else int(enc("True")[0]) if enc else 1
        self.false_id = int(false_id) if false_id is not None else int(enc("False")[0]) if enc else 0

    def _target(self, rng):
        return bool(rng.random() < 0.5)

    def step(self, state: SyntheticState, action_tokens: Sequence[int]):
        first = int(action_tokens[0]) if len(action_tokens) else -1
        want = self.true_id if state.target else self.false_id
        r = 1.0 if first == want else 0.0
        return state, [], r, True, {"label": bool(state.target), "first_token": first, "final_reward": r}


class SyntheticParityEnv(_SyntheticBase):
    def __init__(self, tokenizer, **kw):
        kw.setdefault("image_size", 64)
        kw.setdefault("prompt_tokens", 16)
        super().__init__(tokenizer, **kw)
        self.tokens_per_action = 16

    def _target(self, rng):
        return None

    def step(self, state: SyntheticState, action_tokens: Sequence[int]):
        first = int(action_tokens[0]) if len(action_tokens) else 1
        r = 1.0 if first % 2 == 0 else 0.0
        return state, [], r, True, {"first_token": first, "final_reward": r}


__all__ = ["SyntheticPrompt", "SyntheticState", "SyntheticGeoEnv", "SyntheticTrueFalseEnv",
           "SyntheticParityEnv", "sphere_point"]
