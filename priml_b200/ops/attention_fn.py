"""Autograd function over the tcgen05 flash-attention kernels."""

from __future__ import annotations

import torch
from torch import Tensor

from priml_b200.ops._loader import native


def _prep(t: Tensor) -> Tensor:
    """Kernel needs heads x head_dim contiguous and 16-byte aligned rows; other strides are free."""
    if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1] or t.data_ptr() % 16 or (t.stride(1) * 2) % 16 or (t.stride(0) * 2) % 16:
        return t.contiguous()
    return t


class FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q: Tensor, k: Tensor, v: Tensor, causal: bool, scale: float, window: int) -> Tensor:  # type: ignore[override]
        q, k, v = _prep(q), _prep(k), _prep(v)
        o, lse = native().attn_fwd(q, k, v, scale, causal, window)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale, ctx.window = causal, scale, window
        return o

    @staticmethod
    def backward(ctx, do: Tensor):  # type: ignore[override]
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = native().attn_bwd(q, k, v, o, _prep(do), lse, ctx.scale, ctx.causal, ctx.window)
        return dq, dk, dv, None, None, None
