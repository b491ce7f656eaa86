"""Tensor-like inputs (``priml/math/custom_types.py:74-160``).

``convert_to_tensor`` turns Python scalars, sequences, NumPy arrays and tensors
into tensors that share one dtype and device: the explicit ``dtype`` if given,
otherwise the promotion of the tensor inputs' dtypes (Python numbers adopt it),
otherwise ``dtype_hint``, otherwise the default float dtype.
"""

from __future__ import annotations

from typing import Any, Union, overload

import numpy as np
import torch
from torch import Tensor

__all__ = ["Tensorable", "convert_to_tensor"]

Tensorable = Union[Tensor, np.ndarray, float, int, bool, "list[Any]", "tuple[Any, ...]"]


def _dtype_of(x: Any) -> torch.dtype | None:
    if isinstance(x, Tensor):
        return x.dtype
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.empty(0, dtype=x.dtype)).dtype
    return None


def _device_of(xs: tuple[Any, ...]) -> torch.device | None:
    for x in xs:
        if isinstance(x, Tensor) and x.device.type != "cpu":
            return x.device
    for x in xs:
        if isinstance(x, Tensor):
            return x.device
    return None


@overload
def convert_to_tensor(__x: Tensorable, *, dtype: torch.dtype | None = ..., device: Any = ...,
                      dtype_hint: torch.dtype | None = ...) -> Tensor: ...  # fmt: skip
@overload
def convert_to_tensor(__x: Tensorable, __y: Tensorable, *xs: Tensorable, dtype: torch.dtype | None = ...,
                      device: Any = ..., dtype_hint: torch.dtype | None = ...) -> tuple[Tensor, ...]: ...  # fmt: skip
def convert_to_tensor(*xs: Tensorable, dtype: torch.dtype | None = None, device: Any = None,
                      dtype_hint: torch.dtype | None = None) -> Tensor | tuple[Tensor, ...]:  # fmt: skip
    if dtype is None:
        found = [d for d in (_dtype_of(x) for x in xs) if d is not None]
        if found:
            dtype = found[0]
            for d in found[1:]:
                dtype = torch.promote_types(dtype, d)
            if not dtype.is_floating_point and not dtype.is_complex and any(isinstance(x, float) for x in xs):
                dtype = torch.get_default_dtype()
        elif dtype_hint is not None:
            dtype = dtype_hint
        elif all(isinstance(x, bool) for x in xs):
            dtype = torch.bool
        elif all(isinstance(x, int) and not isinstance(x, bool) for x in xs):
            dtype = torch.get_default_dtype()
        else:
            dtype = torch.get_default_dtype()
    dev = device if device is not None else _device_of(xs)
    out = tuple(torch.as_tensor(x, dtype=dtype, device=dev) for x in xs)
    return out[0] if len(out) == 1 else out
