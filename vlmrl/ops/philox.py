"""Philox-4x32-10 counter-based generator (Salmon et al., SC'11, "Parallel random
numbers: as easy as 1, 2, 3").  NumPy twin of the device implementation in
``csrc/common.cuh`` so the sampler is reproducible on CPU and GPU.

Counter = (row_lo, row_hi, step, 0), key = (seed_lo, seed_hi).  The uniform is
``(x0 >> 8) * 2^-24 + 2^-25``, strictly inside (0, 1).
"""

from __future__ import annotations

import numpy as np

_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32(c0, c1, c2, c3, k0, k1, rounds: int = 10):
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint32) for c in (c0, c1, c2, c3))
    k0, k1 = np.uint32(k0), np.uint32(k1)
    with np.errstate(over="ignore"):
        for _ in range(rounds):
            p0 = _M0 * c0.astype(np.uint64)
            p1 = _M1 * c2.astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & _MASK).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & _MASK).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
            k0 = np.uint32(k0 + _W0)
            k1 = np.uint32(k1 + _W1)
    return c0, c1, c2, c3


def philox_uniform_np(seed: int, rows: np.ndarray, step: int) -> np.ndarray:
    rows = np.asarray(rows, dtype=np.uint64)
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    x0, _, _, _ = philox4x32((rows & _MASK).astype(np.uint32), (rows >> np.uint64(32)).astype(np.uint32),
                             np.full(rows.shape, int(step) & 0xFFFFFFFF, np.uint32), np.zeros(rows.shape, np.uint32),
                             seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    return ((x0 >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24) + np.float32(2.0 ** -25)).astype(np.float32)


__all__ = ["philox4x32", "philox_uniform_np"]
