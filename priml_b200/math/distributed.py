"""Cross-rank log-space reductions (``priml/math/distributed.py:17-78``).

Each rank reduces its own data with ``logsumexp`` over ``dim``, the partial
results are all-gathered, and a second ``logsumexp`` over ranks gives the
global value (``logmeanexp`` subtracts the log of the global element count).
Without an initialized process group the local result is returned.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch
import torch.distributed as dist
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor

__all__ = ["logmeanexp_all_to_all", "logsumexp_all_to_all"]


def _reduce(x: Tensorable, dim: int | Sequence[int], keepdim: bool, world_size: int | None, group: object,
            mean: bool) -> Tensor:  # fmt: skip
    x = convert_to_tensor(x)
    local = torch.logsumexp(x, dim=dim, keepdim=keepdim)
    if local.numel() == 0:
        return local
    count = x.numel() // local.numel()
    if dist.is_available() and dist.is_initialized():
        n = world_size if world_size is not None else dist.get_world_size(group)  # type: ignore[arg-type]
        parts = [torch.empty_like(local) for _ in range(n)]
        dist.all_gather(parts, local.contiguous(), group=group)  # type: ignore[arg-type]
        local = torch.logsumexp(torch.stack(parts), dim=0)
        count *= n
    return local - math.log(count) if mean else local


def logsumexp_all_to_all(x: Tensorable, dim: int | Sequence[int] = -1, keepdim: bool = False,
                         world_size: int | None = None, group: object = None) -> Tensor:  # fmt: skip
    return _reduce(x, dim, keepdim, world_size, group, mean=False)


def logmeanexp_all_to_all(x: Tensorable, dim: int | Sequence[int] = -1, keepdim: bool = False,
                          world_size: int | None = None, group: object = None) -> Tensor:  # fmt: skip
    return _reduce(x, dim, keepdim, world_size, group, mean=True)
