"""Flash attention entry point for ``[B, S, H, D]`` tensors with grouped KV heads.

Runs the hand-written tcgen05 kernels (``csrc/attention_*.cu``) for bf16 inputs
with (query/key, value) head dims (64, 64), (128, 128) or (192, 128) -- the last is
multi-head latent attention's 128 + 64 rotary channels with 128 value channels.
Other head dims go through ``torch.nn.functional.scaled_dot_product_attention``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200.ops._loader import native

__all__ = ["flash_attention", "kernel_supports"]


def kernel_supports(q: Tensor, k: Tensor, v: Tensor, window: int | None) -> bool:
    n = native()
    if not hasattr(n, "attn_fwd"):
        return False
    d, dv = q.shape[-1], v.shape[-1]
    return (
        q.dtype == torch.bfloat16
        and k.dtype == torch.bfloat16
        and v.dtype == torch.bfloat16
        and (d, dv) in ((64, 64), (128, 128), (192, 128))
        and q.shape[-2] % k.shape[-2] == 0
    )


def _sdpa(q: Tensor, k: Tensor, v: Tensor, causal: bool, scale: float, window: int | None) -> Tensor:
    qt, kt, vt = (x.transpose(1, 2) for x in (q, k, v))
    mask = None
    if window is not None:
        s, t = q.shape[1], k.shape[1]
        idx = torch.arange(t, device=q.device)
        off = idx[t - s :, None] - idx[None, :]
        mask = (off >= 0) & (off <= window)
        causal = False
    out = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, is_causal=causal, scale=scale, enable_gqa=True)
    return out.transpose(1, 2)


def flash_attention(
    q: Tensor, k: Tensor, v: Tensor, *, causal: bool = True, scale: float | None = None, window: int | None = None
) -> Tensor:
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if q.dtype != torch.bfloat16 and torch.is_autocast_enabled("cuda"):
        q, k, v = (x.to(torch.bfloat16) for x in (q, k, v))
    if kernel_supports(q, k, v, window):
        from priml_b200.ops.attention_fn import FlashAttnFn

        return FlashAttnFn.apply(q, k, v, causal, float(scale), -1 if window is None else int(window))
    return _sdpa(q, k, v, causal, float(scale), window)
