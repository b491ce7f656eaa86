"""Optimizers (``priml/optimizers/__init__.py:14-175``)."""

from __future__ import annotations

import math
from collections.abc import Iterable
from typing import Any, Protocol

import torch

from priml_b200.optimizers.composite import Selector, CompositeOptimizer, complement, everything, excluding, matching
from priml_b200.optimizers.fused_adamw import FusedAdamW
from priml_b200.optimizers.misc import AdamATan2, Newton, SignSGD
from priml_b200.optimizers.muon import (
    Muon,
    NorMuon,
    adjust_lr_conv_heuristic,
    adjust_lr_match_rms_adamw,
    adjust_lr_original,
)

__all__ = [
    "AdamATan2",
    "CompositeOptimizer",
    "FusedAdamW",
    "HasParamGroups",
    "Muon",
    "Newton",
    "NorMuon",
    "Selector",
    "SignSGD",
    "adjust_lr_conv_heuristic",
    "adjust_lr_match_rms_adamw",
    "adjust_lr_original",
    "apply_lr_scale",
    "clip_grad_norm",
    "complement",
    "everything",
    "excluding",
    "lr_scale",
    "matching",
    "remember_initial_lrs",
    "step_optimizers",
    "zero_optimizers",
]


class HasParamGroups(Protocol):
    param_groups: list[dict[str, Any]]


def lr_scale(step: int, total_steps: int, warmup_steps: int = 0, min_ratio: float = 0.0) -> float:
    """Linear warmup then cosine decay to ``min_ratio`` (held past ``total_steps``)."""
    if step < warmup_steps:
        return step / max(1, warmup_steps)
    progress = min(1.0, (step - warmup_steps) / max(1, total_steps - warmup_steps))
    return min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * progress))


def remember_initial_lrs(optimizers: Iterable[HasParamGroups]) -> None:
    for o in optimizers:
        for g in o.param_groups:
            g.setdefault("initial_lr", g["lr"])


def apply_lr_scale(optimizers: Iterable[HasParamGroups], scale: float) -> None:
    for o in optimizers:
        for g in o.param_groups:
            g["lr"] = g.get("initial_lr", g["lr"]) * scale


def step_optimizers(optimizers: Iterable[torch.optim.Optimizer]) -> None:
    for o in optimizers:
        o.step()


def zero_optimizers(optimizers: Iterable[torch.optim.Optimizer], set_to_none: bool = True) -> None:
    for o in optimizers:
        o.zero_grad(set_to_none=set_to_none)


def clip_grad_norm(parameters: Iterable[torch.Tensor], max_norm: float | None) -> torch.Tensor | None:
    if max_norm is None or math.isinf(max_norm):
        return None
    return torch.nn.utils.clip_grad_norm_(list(parameters), max_norm)
