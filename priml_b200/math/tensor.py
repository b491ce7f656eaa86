"""Tensor utilities (``priml/math/tensor.py:19-170``)."""

from __future__ import annotations

from collections.abc import Sequence
from typing import Literal

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor

__all__ = ["as_batch_tensor", "compiled_scale_and_shift", "pad", "scale_and_shift",
           "warmup_compiled_scale_and_shift"]  # fmt: skip


def pad(input: Tensorable, pad: Sequence[int],  # noqa: A002
        mode: Literal["reflect", "replicate", "circular", "constant", "reflect_replicate"] = "constant",
        value: float | None = None) -> Tensor:  # fmt: skip
    """``F.pad`` plus ``"reflect_replicate"``: reflection that never fails on short axes.

    Reflecting by ``r`` needs ``r <= size - 1``. For each side, first replicate
    ``c = max(0, ceil((r + 1 - size) / 2))`` edge values, then reflect the other
    ``r - c``: the axis has grown to ``size + c``, and ``r - c <= size + c - 1``.
    """
    x = convert_to_tensor(input).contiguous()
    squeeze = x.ndim < 2
    if squeeze:
        x = x[None]
    if mode != "reflect_replicate":
        y = F.pad(x, list(pad), mode=mode, value=value)
        return y[0] if squeeze else y
    pads = list(pad)
    rank = len(pads) // 2
    sizes = [x.shape[-1 - (i // 2)] for i in range(2 * rank)]
    rep = [min(r, max(0, -((size - r - 1) // 2))) for r, size in zip(pads, sizes, strict=True)]
    ref = [r - c for r, c in zip(pads, rep, strict=True)]
    if any(rep):
        x = F.pad(x, rep, mode="replicate")
    y = F.pad(x, ref, mode="reflect") if any(ref) else x
    return y[0] if squeeze else y


def scale_and_shift(x: Tensor, shift: Tensor, scale: Tensor) -> Tensor:
    """``x.to(scale.dtype) * scale + shift`` (e.g. uint8 pixels -> normalized bf16)."""
    return torch.addcmul(shift, x.to(scale.dtype), scale)


# The same op under the reference's name; one fused addcmul needs no compilation.
compiled_scale_and_shift = scale_and_shift


def warmup_compiled_scale_and_shift(dtype_in: torch.dtype = torch.uint8, dtype_out: torch.dtype = torch.bfloat16) -> None:
    """Nothing to warm up (kept for API compatibility)."""
    del dtype_in, dtype_out


def as_batch_tensor(x: Tensorable, min_ndim: int = 4, max_ndim: int = 5, dtype: torch.dtype | None = None,
                    device: torch.device | str | None = None) -> Tensor:  # fmt: skip
    """Left-pad the shape with ones up to ``min_ndim`` dims; flatten leading dims down to ``max_ndim``."""
    t = convert_to_tensor(x, dtype=dtype, device=device) if not isinstance(x, Tensor) else x.to(dtype=dtype or x.dtype, device=device or x.device)
    if t.ndim < min_ndim:
        t = t.reshape((1,) * (min_ndim - t.ndim) + tuple(t.shape))
    if t.ndim > max_ndim:
        keep = max_ndim - 1
        t = t.reshape(-1, *t.shape[t.ndim - keep :])
    return t
