"""Loss math (``priml/math/loss.py:23-165``)."""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

__all__ = ["cross_entropy_with_batched_smoothing", "log_stablemax", "stablemax_cross_entropy"]


def cross_entropy_with_batched_smoothing(
    logits: Tensor, targets: Tensor, smoothing: Tensor | float = 0.0, *, ignore_index: int = -100
) -> Tensor:
    """Unreduced CE where label smoothing may differ per example (``smoothing`` broadcast to ``targets``)."""
    logp = F.log_softmax(logits.float(), dim=-1)
    valid = targets != ignore_index
    t = targets.clamp_min(0)
    nll = -logp.gather(-1, t.unsqueeze(-1)).squeeze(-1)
    smooth = -logp.mean(dim=-1)
    eps = torch.as_tensor(smoothing, dtype=logp.dtype, device=logp.device)
    return torch.where(valid, (1 - eps) * nll + eps * smooth, torch.zeros_like(nll))


def _s(x: Tensor) -> Tensor:
    return torch.where(x < 0, 1 / (1 - x), x + 1)


def log_stablemax(x: Tensor, dim: int = -1) -> Tensor:
    """``log(s(x) / sum s(x))`` with ``s(x) = x+1 (x>=0), 1/(1-x) (x<0)`` (Prieto et al. 2025)."""
    s = _s(x.double() if x.dtype == torch.float64 else x.float())
    return torch.log(s / s.sum(dim=dim, keepdim=True))


def stablemax_cross_entropy(logits: Tensor, targets: Tensor, *, ignore_index: int = -100) -> Tensor:
    logp = log_stablemax(logits.to(torch.float64), dim=-1)
    valid = targets != ignore_index
    nll = -logp.gather(-1, targets.clamp_min(0).unsqueeze(-1).long()).squeeze(-1)
    return torch.where(valid, nll, torch.zeros_like(nll)).to(logits.dtype if logits.is_floating_point() else torch.float32)
