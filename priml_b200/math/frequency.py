"""Discrete cosine transforms (``priml/math/frequency.py:20-175``).

DCT-II with SciPy's conventions: unnormalized
``X_k = 2 sum_n x_n cos(pi k (2n + 1) / (2N))``; ``normalize=True`` is the
orthonormal transform. Both directions are one matrix product against a cached
cosine basis (fp64-built, cast to the input dtype): for the transform lengths
used on images and sequences the GEMM is exact to rounding and runs on the
tensor cores, with no FFT reordering.
"""

from __future__ import annotations

import functools
import math
from collections.abc import Sequence

import torch
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor

__all__ = ["dct1d", "dctnd", "idct1d", "idctnd"]


@functools.lru_cache(maxsize=64)
def _basis(n: int, normalize: bool, inverse: bool, dtype: torch.dtype, device: str) -> Tensor:
    k = torch.arange(n, dtype=torch.float64)
    c = torch.cos(math.pi * k[:, None] * (2 * k[None, :] + 1) / (2 * n))  # [k, n]
    if normalize:
        scale = torch.full((n,), math.sqrt(2.0 / n), dtype=torch.float64)
        scale[0] = math.sqrt(1.0 / n)
        fwd = c * scale[:, None]  # orthonormal: inverse is the transpose
        m = fwd.T if inverse else fwd
    elif inverse:
        # x_n = X_0 / (2N) + (1/N) sum_{k>=1} X_k cos(...)
        w = torch.full((n,), 1.0 / n, dtype=torch.float64)
        w[0] = 0.5 / n
        m = (c * w[:, None]).T
    else:
        m = 2.0 * c
    return m.to(dtype=dtype, device=device)


def _apply(x: Tensor, dim: int, normalize: bool, inverse: bool) -> Tensor:
    n = x.shape[dim]
    dt = x.dtype if x.is_floating_point() else torch.get_default_dtype()
    mat = _basis(n, normalize, inverse, dt, str(x.device))
    y = torch.movedim(x.to(dt), dim, -1) @ mat.T
    return torch.movedim(y, -1, dim)


def dct1d(x: Tensorable, *, normalize: bool = False) -> Tensor:
    """DCT-II over the last dimension."""
    return _apply(convert_to_tensor(x), -1, normalize, inverse=False)


def idct1d(x: Tensorable, *, normalize: bool = False) -> Tensor:
    """Inverse of :func:`dct1d` (a scaled DCT-III): ``idct1d(dct1d(x)) == x``."""
    return _apply(convert_to_tensor(x), -1, normalize, inverse=True)


def _axes(x: Tensor, axis: int | Sequence[int] | None) -> tuple[int, ...]:
    if axis is None:
        return tuple(range(x.ndim))
    return tuple(a % x.ndim for a in ((axis,) if isinstance(axis, int) else axis))


def dctnd(x: Tensorable, *, axis: int | Sequence[int] | None = None, normalize: bool = False) -> Tensor:
    """Separable DCT-II over ``axis`` (all axes when None)."""
    t = convert_to_tensor(x)
    for a in _axes(t, axis):
        t = _apply(t, a, normalize, inverse=False)
    return t


def idctnd(x: Tensorable, *, axis: int | Sequence[int] | None = None, normalize: bool = False) -> Tensor:
    t = convert_to_tensor(x)
    for a in _axes(t, axis):
        t = _apply(t, a, normalize, inverse=True)
    return t
