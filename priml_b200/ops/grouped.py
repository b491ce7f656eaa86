"""Grouped expert MLP over expert-sorted rows.

``x_sorted`` rows ``offsets[e]:offsets[e+1]`` belong to expert ``e``; up
weights ``[E, 2H, C]`` (gate rows first), down weights ``[E, C, H]``.
"""

from __future__ import annotations

from torch import Tensor

from priml_b200.ops import functional as fn


def grouped_swiglu_mlp(x_sorted: Tensor, up_w: Tensor, down_w: Tensor, offsets: Tensor) -> Tensor:
    bounds = offsets.tolist()
    pieces = []
    for e in range(up_w.shape[0]):
        lo, hi = bounds[e], bounds[e + 1]
        if hi > lo:
            h = fn.linear_swiglu(x_sorted[lo:hi], up_w[e])
            pieces.append(fn.linear(h, down_w[e]))
    if not pieces:
        return x_sorted.new_zeros(0, down_w.shape[1])
    import torch

    return torch.cat(pieces, dim=0)
