"""Adaptive KL coefficient controller (reference ``core/kl.py:12-39``).

Above ``2*target`` the coefficient grows by ``rate`` (from 0 it jumps to
``min(1e-4, coef_max)``); below ``target/2`` it shrinks by ``rate`` (staying 0
at 0); beyond ``max(0.5, 5*target)`` it is additionally multiplied by
``rate**2``; the result is clamped to ``[coef_min, coef_max]``.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class AdaptiveKL:
    target: float = 0.02
    rate: float = 1.5
    coef_min: float = 1e-5
    coef_max: float = 0.5

    def _clamp(self, c: float) -> float:
        return min(self.coef_max, max(self.coef_min, c))

    def update(self, approx_kl: float, current_coef: float) -> float:
        c = float(current_coef)
        if self.target <= 0:
            return self._clamp(c)
        if approx_kl > 2.0 * self.target:
            c = c * self.rate if c > 0 else min(1e-4, self.coef_max)
        elif approx_kl < 0.5 * self.target:
            c = c / self.rate if c > 0 else 0.0
        if approx_kl > max(0.5, 5.0 * self.target):
            c *= self.rate ** 2
        return self._clamp(c)


__all__ = ["AdaptiveKL"]
