"""Counter-based RNG helpers.

``RngSeq`` mirrors reference ``utils/rng.py:12-21`` (``RngSeq(seed).next()`` hands
out a fresh, independent key per call).  Keys here are 64-bit integers derived
with SplitMix64, and every GPU random draw (sampler, synthetic data) is a pure
function of (key, counter) through Philox-4x32 inside the kernels, so results
do not depend on launch order or on the number of ranks.
"""

from __future__ import annotations

from dataclasses import dataclass, field

_MASK64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & _MASK64
    z = x
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK64
    return z ^ (z >> 31)


def fold_in(key: int, data: int) -> int:
    """Derive a child key from ``key`` and an integer tag (rank, step, row ...)."""
    return splitmix64((int(key) ^ splitmix64(int(data) & _MASK64)) & _MASK64)


@dataclass
class RngSeq:
    seed: int
    _state: int = field(init=False, repr=False)

    def __post_init__(self) -> None:
        self._state = splitmix64(int(self.seed) & _MASK64)

    def next(self) -> int:
        self._state = splitmix64(self._state)
        return self._state & ((1 << 63) - 1)

    def state(self) -> int:
        """The generator position (for checkpoints)."""
        return int(self._state)

    def set_state(self, state: int) -> None:
        self._state = int(state) & _MASK64


__all__ = ["RngSeq", "fold_in", "splitmix64"]
