"""Learning-rate multipliers as functions of progress in [0, 1]
(``priml/math/schedules.py:49-322``). A schedule maps the fraction of the
budget spent to a multiplier of each group's ``initial_lr``."""

from __future__ import annotations

import math
from collections.abc import Callable

__all__ = [
    "constant",
    "cosine",
    "cosine_restarts",
    "exponential",
    "linear",
    "multiply_schedules",
    "one_cycle",
    "polynomial",
    "staircase",
    "trapezoidal",
    "warmup",
]

Schedule = Callable[[float], float]


def _clamped(progress: float) -> float:
    return min(1.0, max(0.0, float(progress)))


def multiply_schedules(*schedules: Schedule) -> Schedule:
    """Pointwise product of schedules (e.g. a warmup factor times a decay)."""

    def product(progress: float) -> float:
        out = 1.0
        for s in schedules:
            out *= s(progress)
        return out

    return product


def constant(progress: float) -> float:
    del progress
    return 1.0


def linear(progress: float, *, final: float = 0.0) -> float:
    return 1.0 + (final - 1.0) * _clamped(progress)


def polynomial(progress: float, *, power: float = 1.0) -> float:
    return math.pow(1.0 - _clamped(progress), power)


def cosine(progress: float, *, final: float = 0.0) -> float:
    return final + (1.0 - final) * 0.5 * (1.0 + math.cos(math.pi * _clamped(progress)))


def exponential(progress: float, *, decay: float) -> float:
    """Geometric decay reaching ``decay`` at the end of the run."""
    if decay <= 0:
        raise ValueError(f"decay must be positive; got {decay}.")
    return math.pow(decay, _clamped(progress))


def staircase(progress: float, *, drops: int = 3, gamma: float = 0.1) -> float:
    """``drops`` equal-width steps, each multiplying by ``gamma``."""
    if drops < 0:
        raise ValueError(f"drops must be nonnegative; got {drops}.")
    if drops == 0:
        return 1.0
    return math.pow(gamma, min(int(_clamped(progress) * (drops + 1)), drops))


def warmup(progress: float, *, fraction: float) -> float:
    """Linear ramp over the first ``fraction`` of the run, then 1."""
    if fraction <= 0:
        return 1.0
    return min(1.0, _clamped(progress) / fraction)


def trapezoidal(progress: float, *, flat: float = 0.5, final: float = 0.0, cooldown_cosine: bool = False) -> float:
    """Full rate for ``flat`` of the run, then linear (or cosine) to ``final``."""
    if not 0.0 <= flat < 1.0:
        raise ValueError(f"flat must lie in [0, 1); got {flat}.")
    p = _clamped(progress)
    if p < flat:
        return 1.0
    tail = (p - flat) / (1.0 - flat)
    return cosine(tail, final=final) if cooldown_cosine else linear(tail, final=final)


def one_cycle(progress: float, *, warmup_fraction: float = 0.3, initial: float = 0.04, final: float = 0.0) -> float:
    """Cosine rise from ``initial`` to 1 over ``warmup_fraction``, cosine fall to ``final``."""
    if not 0.0 <= warmup_fraction < 1.0:
        raise ValueError(f"warmup_fraction must lie in [0, 1); got {warmup_fraction}.")
    p = _clamped(progress)
    if p < warmup_fraction:
        rising = p / warmup_fraction if warmup_fraction else 1.0
        return initial + (1.0 - initial) * (1.0 - cosine(rising))
    return cosine((p - warmup_fraction) / (1.0 - warmup_fraction), final=final)


def cosine_restarts(progress: float, *, cycles: int = 2, final: float = 0.0, decay: float = 1.0) -> float:
    """``cycles`` cosine anneals; cycle ``i`` peaks at ``decay ** i``."""
    if cycles < 1:
        raise ValueError(f"cycles must be >= 1; got {cycles}.")
    p = _clamped(progress)
    i = min(int(p * cycles), cycles - 1)
    local = p * cycles - i
    return (decay**i) * cosine(local, final=final)
