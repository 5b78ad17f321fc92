"""Model families: ``qwen3vl`` (primary) and ``qwen25vl`` (lazy submodules, reference ``models/__init__.py``)."""

from importlib import import_module


def __getattr__(name):
    if name in ("qwen3vl", "qwen25vl"):
        return import_module(f"vlmrl.models.{name}")
    raise AttributeError(name)


__all__ = ["qwen3vl", "qwen25vl"]
