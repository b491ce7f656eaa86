"""Adaptive average pooling with an optional variance-preserving scale
(``priml/math/pooling.py:20-200``).

Window ``i`` of an axis of length ``S`` pooled to ``O`` covers
``[floor(i S / O), ceil((i + 1) S / O))`` (PyTorch's adaptive rule). With
``variance_preserving`` the window mean is multiplied by ``sqrt(window size)``,
i.e. the output is ``sum / sqrt(size)``: pooling i.i.d. unit-variance inputs
then keeps unit variance. Windows are summed through a cumulative sum along
each pooled axis, so ragged windows cost the same as even ones.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

__all__ = ["adaptive_avg_pool2d", "adaptive_avg_pool3d"]


def _window_sum(x: Tensor, dim: int, out: int) -> tuple[Tensor, Tensor]:
    size = x.shape[dim]
    i = torch.arange(out, device=x.device)
    start = torch.div(i * size, out, rounding_mode="floor")
    end = torch.div((i + 1) * size + out - 1, out, rounding_mode="floor")
    csum = torch.cumsum(x, dim=dim)
    csum = torch.cat([torch.zeros_like(csum.narrow(dim, 0, 1)), csum], dim=dim)
    s = csum.index_select(dim, end) - csum.index_select(dim, start)
    return s, (end - start).to(x.dtype)


def _adaptive(x: Tensor, output_size: tuple[int, ...], variance_preserving: bool) -> Tensor:
    n = len(output_size)
    if any(s == 0 for s in x.shape[-n:]):
        raise ValueError(f"expected non-zero spatial dims, got shape {tuple(x.shape)}")
    if not variance_preserving:
        return (F.adaptive_avg_pool2d if n == 2 else F.adaptive_avg_pool3d)(x, output_size)
    if all(s % o == 0 for s, o in zip(x.shape[-n:], output_size, strict=True)):
        k = tuple(s // o for s, o in zip(x.shape[-n:], output_size, strict=True))
        pool = F.avg_pool2d if n == 2 else F.avg_pool3d
        return pool(x, k, k) * math.sqrt(math.prod(k))
    y = x.float()
    counts = []
    for j, o in enumerate(output_size):
        dim = x.ndim - n + j
        y, c = _window_sum(y, dim, o)
        counts.append(c)
    size = counts[0]
    for c in counts[1:]:
        size = size[..., None] * c
    return (y / torch.sqrt(size)).to(x.dtype)


def adaptive_avg_pool2d(input: Tensor, output_size: tuple[int, int], variance_preserving: bool = False) -> Tensor:  # noqa: A002
    if input.ndim not in (3, 4):
        raise ValueError(f"expected a 3D or 4D tensor, got {input.ndim}D")
    return _adaptive(input, tuple(output_size), variance_preserving)


def adaptive_avg_pool3d(input: Tensor, output_size: tuple[int, int, int], variance_preserving: bool = False) -> Tensor:  # noqa: A002
    if input.ndim not in (4, 5):
        raise ValueError(f"expected a 4D or 5D tensor, got {input.ndim}D")
    return _adaptive(input, tuple(output_size), variance_preserving)
