"""Minibatch slicing (reference ``core/minibatch.py:16-48``).

``shard_for_minibatch`` reshapes a leading dimension ``N`` into ``[chunks, mb]``
(``chunks = max(1, N // mb)``; the tail beyond ``chunks*mb`` is dropped, as in
the reference).  ``minibatch_indices`` is the explicit alternative used by the
trainer: exactly ``n_minibatches`` contiguous, group-aligned index ranges.
"""

from __future__ import annotations

from typing import List, Sequence

import numpy as np
import torch

from vlmrl.models.qwen3vl.model import VisionEmbeddings


def _trim(x, mb: int):
    if mb <= 0:
        raise ValueError("minibatch size must be positive")
    chunks = max(1, int(x.shape[0]) // mb)
    return x[:chunks * mb], chunks


def shard_for_minibatch(x, mb: int):
    if isinstance(x, VisionEmbeddings):
        toks, chunks = _trim(x.tokens, mb)
        deep = tuple(d[:chunks * mb].reshape(chunks, mb, *d.shape[1:]) for d in x.deepstack)
        return VisionEmbeddings(tokens=toks.reshape(chunks, mb, *toks.shape[1:]), deepstack=deep)
    xt, chunks = _trim(x, mb)
    return xt.reshape(chunks, mb, *xt.shape[1:])


def minibatch_indices(n: int, n_minibatches: int, group_size: int = 1) -> List[np.ndarray]:
    """Split ``range(n)`` into ``n_minibatches`` contiguous parts on group boundaries."""
    groups = n // max(1, group_size)
    if groups * group_size != n:
        groups, group_size = n, 1
    k = max(1, min(n_minibatches, groups))
    bounds = np.linspace(0, groups, k + 1).round().astype(int) * group_size
    return [np.arange(bounds[i], bounds[i + 1]) for i in range(k) if bounds[i + 1] > bounds[i]]


__all__ = ["shard_for_minibatch", "minibatch_indices"]
