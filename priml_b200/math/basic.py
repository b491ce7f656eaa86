"""Small numeric helpers (``priml/math/basic.py``)."""

from __future__ import annotations

import math
from collections.abc import Sequence
from typing import Any

import torch
from torch import Tensor

__all__ = ["argsort", "broadcast_sequences", "ceil_div", "ceil_multiple", "factors", "floor_multiple"]


def factors(n: int) -> tuple[int, ...]:
    """Sorted positive divisors of ``n``."""
    if n < 1:
        raise ValueError(f"n must be positive, got {n}")
    small = [d for d in range(1, math.isqrt(n) + 1) if n % d == 0]
    return tuple(sorted(set(small + [n // d for d in small])))


def _to_multiple(x: Any, multiple: float | None, up: bool) -> Any:
    if multiple is None:
        return x
    if isinstance(x, Tensor):
        q = torch.ceil(x / multiple) if up else torch.floor(x / multiple)
        return q * multiple
    q = math.ceil(x / multiple) if up else math.floor(x / multiple)
    return type(multiple)(q * multiple)


def ceil_multiple(x: Any, multiple: float | None) -> Any:
    """Smallest multiple of ``multiple`` that is ``>= x``."""
    return _to_multiple(x, multiple, True)


def floor_multiple(x: Any, multiple: float | None) -> Any:
    """Largest multiple of ``multiple`` that is ``<= x``."""
    return _to_multiple(x, multiple, False)


def ceil_div(x: int, y: int) -> int:
    return -(-x // y)


def argsort(seq: Sequence[Any], *, reverse: bool = False) -> list[int]:
    return sorted(range(len(seq)), key=lambda i: seq[i], reverse=reverse)


def broadcast_sequences(*args: Any) -> tuple[list[Any], ...]:
    """Broadcast scalars / length-1 sequences against sequences of length n."""
    lists = [list(a) if isinstance(a, Sequence) and not isinstance(a, str) else [a] for a in args]
    n = max(len(a) for a in lists)
    for a in lists:
        if len(a) not in (1, n):
            raise ValueError(f"Incompatible lengths: {[len(x) for x in lists]}.")
    return tuple(a * n if len(a) == 1 else a for a in lists)
