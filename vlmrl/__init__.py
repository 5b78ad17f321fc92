"""vlmrl — a Blackwell-native (sm_100a) reinforcement-learning framework for vision-language models.

Public module layout follows the reference project's ``vlmrl.*`` namespace
(reference ``pyproject.toml:46-51``): ``vlmrl.core`` (RL algorithms, sampler,
rollout, trainer and eval CLIs), ``vlmrl.envs`` (BaseEnv environments),
``vlmrl.models`` (Qwen3-VL / Qwen2.5-VL), ``vlmrl.utils`` (checkpoint, train
state, image/prompt helpers).  B200-specific layers are ``vlmrl.ops`` (the
hand-written CUDA kernels and their PyTorch oracles) and ``vlmrl.parallel``
(process groups, FSDP / TP engines, NVLink peer-memory collectives).

Submodules load lazily so ``import vlmrl`` stays cheap.
"""

from importlib import import_module

__version__ = "0.1.0"

_SUBMODULES = ("core", "envs", "models", "ops", "parallel", "utils")


def __getattr__(name):
    if name in _SUBMODULES:
        return import_module(f"vlmrl.{name}")
    raise AttributeError(f"module 'vlmrl' has no attribute {name!r}")


__all__ = list(_SUBMODULES)
