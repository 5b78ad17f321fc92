"""Environment protocol, registry and factory.

API parity with reference ``envs/base.py:10-113``:

* ``BaseState.render()``; ``BaseEnv`` with class attributes
  ``tokens_per_action=32``, ``force_answer_at=-1``, ``num_tasks=-1``;
* ``reset(idx) -> (state, obs)`` and
  ``step(state, action_tokens) -> (state, out_tokens, reward, done, info)``;
* ``clean_action`` keeps tokens up to and including the first EOS;
* ``step_list`` is the vectorised wrapper (info values collected per key);
* ``create_env(name, tokenizer, **kw)`` with the same aliases
  (nlvr2/truefalse, vision/vision_caption/caption, geospot) plus the synthetic
  benchmark environments of this framework.
"""

from __future__ import annotations

from dataclasses import dataclass
from importlib import import_module
from typing import Any, Dict, List, Optional, Sequence, Tuple


@dataclass(frozen=True)
class BaseState:
    def render(self) -> str:
        raise NotImplementedError


class BaseEnv:
    tokens_per_action: int = 32
    force_answer_at: int = -1
    num_tasks: int = -1

    def reset(self, idx: int) -> Tuple[BaseState, Any]:
        raise NotImplementedError

    def step(self, state: BaseState, action_tokens: Sequence[int]) -> Tuple[BaseState, Sequence[int], float, bool, Dict[str, Any]]:
        raise NotImplementedError

    @staticmethod
    def clean_action(action_tokens: Sequence[int], end_token: int) -> List[int]:
        out = []
        for tok in action_tokens:
            out.append(int(tok))
            if int(tok) == int(end_token):
                break
        return out

    def step_list(self, states: Sequence[BaseState], actions: Sequence[Sequence[int]]):
        if len(states) != len(actions):
            raise ValueError(f"states/actions length mismatch: {len(states)} vs {len(actions)}")
        new_states, outputs, rewards, dones = [], [], [], []
        info: Dict[str, List[Any]] = {}
        for st, act in zip(states, actions):
            s2, out, r, d, extra = self.step(st, act)
            new_states.append(s2)
            outputs.append(out)
            rewards.append(float(r))
            dones.append(bool(d))
            for k, v in extra.items():
                info.setdefault(k, []).append(v)
        return new_states, outputs, rewards, dones, info


def resolve_eos_id(tokenizer) -> Optional[int]:
    eos = getattr(tokenizer, "eos_token_id", None)
    if eos is not None:
        return int(eos)
    getter = getattr(tokenizer, "get_eos_token_id", None)
    return int(getter()) if callable(getter) and getter() is not None else None


_ENV_REGISTRY: Dict[str, Tuple[str, str]] = {
    "nlvr2": ("vlmrl.envs.nlvr2", "NLVR2Env"),
    "truefalse": ("vlmrl.envs.nlvr2", "NLVR2Env"),
    "vision": ("vlmrl.envs.vision_caption", "VisionCaptionEnv"),
    "vision_caption": ("vlmrl.envs.vision_caption", "VisionCaptionEnv"),
    "caption": ("vlmrl.envs.vision_caption", "VisionCaptionEnv"),
    "geospot": ("vlmrl.envs.geospot", "GeospotEnv"),
    # synthetic, offline benchmark environments (no dataset download)
    "synthetic_geo": ("vlmrl.envs.synthetic", "SyntheticGeoEnv"),
    "synthetic_truefalse": ("vlmrl.envs.synthetic", "SyntheticTrueFalseEnv"),
    "synthetic_parity": ("vlmrl.envs.synthetic", "SyntheticParityEnv"),
}


def register_env(name: str, module_path: str, attr: str) -> None:
    _ENV_REGISTRY[name.strip().lower()] = (module_path, attr)


def create_env(env_name: str, tokenizer, **env_kwargs) -> BaseEnv:
    key = env_name.strip().lower()
    if key not in _ENV_REGISTRY:
        raise ValueError(f"Unknown environment name: {env_name!r}")
    module_path, attr = _ENV_REGISTRY[key]
    return getattr(import_module(module_path), attr)(tokenizer, **env_kwargs)


__all__ = ["BaseState", "BaseEnv", "create_env", "register_env", "resolve_eos_id"]
