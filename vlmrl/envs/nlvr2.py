"""NLVR2 two-image True/False reasoning (reference ``envs/nlvr2.py:24-128``).

Reward is 1 when the parsed answer equals the label.  Parsing: "true"/"false"
when exactly one of them occurs, else "yes"/"no" likewise, else False.
The dataset comes from the local HF datasets cache (``HuggingFaceM4/NLVR2``)
or from an explicit ``samples`` list.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, List, Optional, Sequence

from vlmrl.envs.base import BaseEnv, BaseState, resolve_eos_id
from vlmrl.utils.vlm import decode_tokens


@dataclass(frozen=True)
class NLVR2Sample:
    statement: str
    image_left: Any
    image_right: Any
    label: bool


@dataclass(frozen=True)
class NLVR2Prompt:
    statement: str
    image_left: Any
    image_right: Any
    label: bool


@dataclass(frozen=True)
class NLVR2State(BaseState):
    dataset_idx: int
    sample: NLVR2Sample

    def render(self) -> str:
        return f"Look at the two images. {self.sample.statement} True or False?"


def parse_binary(text: str) -> bool:
    t = text.lower().strip()
    for pos, neg in (("true", "false"), ("yes", "no")):
        has_pos, has_neg = pos in t, neg in t
        if has_pos != has_neg:
            return has_pos
    return False


class NLVR2Env(BaseEnv):
    def __init__(self, tokenizer, split: str = "validation", samples: Optional[List[NLVR2Sample]] = None):
        super().__init__()
        self.tokenizer = tokenizer
        self.tokens_per_action = 128
        self.split = split
        self.dataset = samples if samples is not None else self._load_dataset(split)
        self.num_tasks = len(self.dataset)
        self.eos_token_id = resolve_eos_id(tokenizer)

    @staticmethod
    def _load_dataset(split: str) -> List[NLVR2Sample]:
        from datasets import load_dataset

        rows = load_dataset("HuggingFaceM4/NLVR2", split=split)
        return [NLVR2Sample(r["sentence"], r["left_image"], r["right_image"], bool(r["label"])) for r in rows]

    def reset(self, idx: int):
        i = idx % len(self.dataset)
        s = self.dataset[i]
        return NLVR2State(dataset_idx=i, sample=s), NLVR2Prompt(s.statement, s.image_left, s.image_right, s.label)

    _parse_binary = staticmethod(parse_binary)

    def step(self, state: NLVR2State, action_tokens: Sequence[int]):
        if self.eos_token_id is not None:
            action_tokens = self.clean_action(action_tokens, self.eos_token_id)
        text = decode_tokens(self.tokenizer, action_tokens).strip().lower()
        pred = parse_binary(text)
        reward = 1.0 if pred == state.sample.label else 0.0
        return state, [], reward, True, {"response": text, "predicted": pred, "label": state.sample.label}


__all__ = ["NLVR2Sample", "NLVR2Prompt", "NLVR2State", "NLVR2Env", "parse_binary"]
