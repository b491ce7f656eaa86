"""Activations (``priml/math/activations.py:17``)."""

from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["relu_squared"]


def relu_squared(x: Tensor) -> Tensor:
    """``relu(x)^2`` (So et al. 2021, Primer); its derivative ``2 relu(x)`` is itself a rectifier."""
    r = torch.relu(x)
    return r * r
