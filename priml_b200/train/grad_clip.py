"""Gradient-norm helpers (``priml/train/grad_clip.py:34-143``).

``fused_grad_norm_clip`` computes the global L2 norm of every gradient a
:class:`FusedAdamW` owns with one multi-tensor kernel per group and returns
``(norm, clip_coefficient)`` as device scalars -- nothing is read back to the
host, so clipping costs no synchronization. Under data/fully-sharded
parallelism the squared norm is all-reduced across ranks first.
"""

from __future__ import annotations

import math
from collections.abc import Iterable

import torch
import torch.distributed as dist
from torch import Tensor

__all__ = ["clip_grad_norm_", "fused_grad_norm_clip", "grad_norm", "total_norm"]


def _local(t: Tensor) -> Tensor:
    return t._local_tensor if hasattr(t, "_local_tensor") else t  # noqa: SLF001


def grad_norm(parameters: Iterable[Tensor]) -> Tensor:
    """Global gradient L2 norm (foreach, fp32)."""
    grads = [_local(p.grad) for p in parameters if p.grad is not None]
    if not grads:
        return torch.zeros(())
    norms = torch._foreach_norm([g.float() for g in grads])  # noqa: SLF001
    sq = torch.stack([n * n for n in norms]).sum()
    if dist.is_available() and dist.is_initialized() and any(hasattr(p.grad, "_local_tensor") for p in parameters if p.grad is not None):
        dist.all_reduce(sq)
    return sq.sqrt()


total_norm = grad_norm


def clip_grad_norm_(parameters: Iterable[Tensor], max_norm: float) -> Tensor:
    params = [p for p in parameters if p.grad is not None]
    norm = grad_norm(params)
    if math.isinf(max_norm):
        return norm
    coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
    torch._foreach_mul_([_local(p.grad) for p in params], coef.to(params[0].grad.device))  # noqa: SLF001
    return norm


def fused_grad_norm_clip(optimizer: object, max_norm: float) -> tuple[Tensor, Tensor] | None:
    """Device-side (norm, clip) over a FusedAdamW's gradients; None when the
    optimizer cannot take its native path (CPU, non-contiguous grads, ...)."""
    fn = getattr(optimizer, "fused_grad_norm", None)
    return fn(max_norm) if callable(fn) else None
