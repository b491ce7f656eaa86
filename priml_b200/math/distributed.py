"""Cross-rank log-space reductions (``priml/math/distributed.py:17-78``)."""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import Tensor

__all__ = ["logmeanexp_all_to_all", "logsumexp_all_to_all"]


def _gather(x: Tensor, group: object = None) -> Tensor:
    if not (dist.is_available() and dist.is_initialized()):
        return x.unsqueeze(0)
    n = dist.get_world_size(group)  # type: ignore[arg-type]
    out = [torch.empty_like(x) for _ in range(n)]
    dist.all_gather(out, x.contiguous(), group=group)  # type: ignore[arg-type]
    return torch.stack(out)


def logsumexp_all_to_all(x: Tensor, group: object = None) -> Tensor:
    """``log(sum_ranks exp(x))`` elementwise, identical on every rank."""
    return torch.logsumexp(_gather(x, group), dim=0)


def logmeanexp_all_to_all(x: Tensor, group: object = None) -> Tensor:
    g = _gather(x, group)
    return torch.logsumexp(g, dim=0) - math.log(g.shape[0])
