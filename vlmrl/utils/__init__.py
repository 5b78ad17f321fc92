"""Utilities: checkpoint I/O, train state, image/prompt helpers, config flags, logging, RNG (lazy)."""

from importlib import import_module

_SUB = ("checkpoint", "train_state", "vlm", "configs", "wandb", "rng", "sharding", "hf_to_jax", "tokenizer", "profiling")


def __getattr__(name):
    if name in _SUB:
        return import_module(f"vlmrl.utils.{name}")
    raise AttributeError(name)


__all__ = list(_SUB)
