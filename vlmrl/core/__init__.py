"""RL algorithms, sampler, rollout glue, trainer and eval CLIs (lazy submodules, reference ``core/__init__.py``)."""

from importlib import import_module

_SUB = ("types", "batching", "minibatch", "kl", "policy", "sampling", "rollout", "ppo", "grpo", "train", "eval", "trainer")


def __getattr__(name):
    if name in _SUB:
        return import_module(f"vlmrl.core.{name}")
    raise AttributeError(name)


__all__ = list(_SUB)
