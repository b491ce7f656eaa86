"""Eval metrics with ``reset / update / compute / state_dict`` (``priml/metrics/``)."""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor

from priml_b200.config import Fig

__all__ = ["BinaryAccuracy", "BitsPerByte", "TopK"]


def _reduce(t: Tensor) -> Tensor:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t)
    return t


class TopK:
    class Config(Fig["TopK"]):
        k: int = 1
        prediction_key: str = "prediction"
        target_key: str = "label"

    def __init__(self, config: Config) -> None:
        self.k = config.k
        self.reset()

    def reset(self) -> None:
        self.correct = 0.0
        self.total = 0.0

    def update(self, prediction: Tensor, target: Tensor) -> None:
        top = prediction.topk(self.k, dim=-1).indices
        self.correct += float((top == target.unsqueeze(-1)).any(-1).sum())
        self.total += float(target.numel())

    def compute(self) -> float:
        t = _reduce(torch.tensor([self.correct, self.total], dtype=torch.float64))
        return float(t[0] / t[1]) if t[1] > 0 else math.nan

    def state_dict(self) -> dict[str, Any]:
        return {"correct": self.correct, "total": self.total}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.correct, self.total = float(s["correct"]), float(s["total"])


class BinaryAccuracy(TopK):
    class Config(Fig["BinaryAccuracy"]):
        threshold: float = 0.0

    def __init__(self, config: Config) -> None:  # type: ignore[override]
        self.threshold = config.threshold
        self.reset()

    def update(self, prediction: Tensor, target: Tensor) -> None:
        self.correct += float(((prediction > self.threshold) == (target > 0.5)).sum())
        self.total += float(target.numel())


class BitsPerByte:
    """``sum(nats) / (ln 2 * sum(bytes))``, accumulated in fp64 and all-reduced once
    in ``compute`` (``priml/metrics/bits_per_byte.py:35-133``)."""

    class Config(Fig["BitsPerByte"]):
        pass

    def __init__(self, config: Config | None = None) -> None:
        del config
        self.reset()

    def reset(self) -> None:
        self.nats = 0.0
        self.bytes = 0.0

    def update(self, token_nats: Tensor, token_bytes: Tensor) -> None:
        keep = token_bytes > 0
        self.nats += float(token_nats.double()[keep].sum())
        self.bytes += float(token_bytes.double()[keep].sum())

    def compute(self) -> float:
        t = _reduce(torch.tensor([self.nats, self.bytes], dtype=torch.float64))
        return float(t[0] / (math.log(2) * t[1])) if t[1] > 0 else math.nan

    def state_dict(self) -> dict[str, Any]:
        return {"nats": self.nats, "bytes": self.bytes}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.nats, self.bytes = float(s["nats"]), float(s["bytes"])
