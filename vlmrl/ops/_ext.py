"""Loader of the native extension ``vlmrl._C`` (built in-tree by ``setup.py build_ext --inplace``).

``ext()`` returns the module or raises with build instructions: ops on CUDA
tensors never fall back to PyTorch.  ``has_ext()`` reports availability, and
``loaded_path()`` the ``.so`` that was imported.
"""

from __future__ import annotations

import importlib

_MOD = None
_ERR = None


def _load():
    global _MOD, _ERR
    if _MOD is not None or _ERR is not None:
        return _MOD
    try:
        import torch  # noqa: F401  (libtorch symbols must be loaded first)

        _MOD = importlib.import_module("vlmrl._C")
    except ImportError as exc:  # not built on this machine
        _ERR = exc
    return _MOD


def has_ext() -> bool:
    return _load() is not None


def ext():
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "vlmrl CUDA extension (vlmrl._C) is not built; run `python setup.py build_ext --inplace` "
            f"(or __graft_entry__.build()). Import error: {_ERR}")
    return mod


def loaded_path() -> str:
    mod = _load()
    return getattr(mod, "__file__", "") if mod is not None else ""


__all__ = ["ext", "has_ext", "loaded_path"]
