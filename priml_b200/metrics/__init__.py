"""Eval metrics with ``reset / update / compute / state_dict`` (``priml/metrics/``).

The protocol is the reference's (``priml/metrics/custom_types.py:20-48``): the
loop calls ``update(model_output, **batch)`` once per eval batch with the train
step's ``eval_loss(...)["model"]`` and the batch itself, and ``compute()``
returns a ``{name: value}`` dict, all-reduced across ranks once.
"""

from __future__ import annotations

import math
from dataclasses import field
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor

from priml_b200.config import Fig

__all__ = ["BinaryAccuracy", "BitsPerByte", "MetricProtocol", "TopK"]


class MetricProtocol:
    """``reset()``, ``update(output, **batch)``, ``compute() -> dict``, ``state_dict`` / ``load_state_dict``."""


def _reduce(t: Tensor) -> Tensor:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else t.device
        u = t.to(dev)
        dist.all_reduce(u)
        return u.cpu()
    return t


class TopK:
    """``top{k}`` accuracy of ``[B, C]`` logits against ``label`` (``priml/metrics/topk.py``)."""

    class Config(Fig["TopK"]):
        k_values: list[int] = field(default_factory=lambda: [1, 5])

    def __init__(self, config: Config | None = None) -> None:
        config = config or TopK.Config()
        if not config.k_values:
            raise ValueError("k_values must contain at least one positive integer.")
        self.k_values = list(config.k_values)
        self.reset()

    def reset(self) -> None:
        self.correct = dict.fromkeys(self.k_values, 0)
        self.total = 0

    def update(self, logits: Tensor, label: Tensor | None = None, **_: Any) -> None:
        if label is None:
            raise ValueError("label must be provided")
        num_classes = logits.size(1)
        top = logits.topk(min(max(self.k_values), num_classes), dim=1).indices
        for k in self.k_values:
            self.correct[k] += int((top[:, : min(k, num_classes)] == label.unsqueeze(1)).any(1).sum())
        self.total += int(label.size(0))

    def compute(self) -> dict[str, float]:
        t = _reduce(torch.tensor([self.total, *(self.correct[k] for k in self.k_values)], dtype=torch.float64))
        if t[0] == 0:
            return {f"top{k}": 0.0 for k in self.k_values}
        return {f"top{k}": float(t[i + 1] / t[0]) for i, k in enumerate(self.k_values)}

    def state_dict(self) -> dict[str, Any]:
        return {"correct": dict(self.correct), "total": self.total}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.correct = {int(k): int(v) for k, v in s["correct"].items()}
        self.total = int(s["total"])


class BinaryAccuracy:
    """Accuracy of pre-sigmoid logits ``[B]`` (or ``[B, 1]``) against 0/1 ``label``."""

    class Config(Fig["BinaryAccuracy"]):
        threshold: float = 0.5
        """Probability at or above which a prediction counts as positive."""

    def __init__(self, config: Config | None = None) -> None:
        self.threshold = (config or BinaryAccuracy.Config()).threshold
        self.reset()

    def reset(self) -> None:
        self.correct = 0
        self.total = 0

    def update(self, logits: Tensor, **batch: Any) -> None:
        targets = batch["label"]
        pred = (torch.sigmoid(logits.squeeze(-1)) > self.threshold).to(targets.dtype)
        self.correct += int((pred == targets).sum())
        self.total += int(targets.size(0))

    def compute(self) -> dict[str, float]:
        t = _reduce(torch.tensor([self.correct, self.total], dtype=torch.float64))
        return {"accuracy": float(t[0] / t[1]) if t[1] > 0 else 0.0}

    def state_dict(self) -> dict[str, Any]:
        return {"correct": self.correct, "total": self.total}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.correct, self.total = int(s["correct"]), int(s["total"])


class BitsPerByte:
    """``sum(nats) / (ln 2 * sum(bytes))`` over scored tokens (``priml/metrics/bits_per_byte.py:35-133``).

    ``update(per_token_nats [B, S], label=..., token_bytes=..., valid_count=...)``: rows past
    ``valid_count`` are padding and skipped; tokens whose byte length is zero (reserved tokens)
    are excluded from both sums. Accumulated in fp64 and all-reduced once in ``compute``.
    """

    class Config(Fig["BitsPerByte"]):
        pass

    def __init__(self, config: Config | None = None) -> None:
        del config
        self.reset()

    def reset(self) -> None:
        self.nats = 0.0
        self.bytes = 0

    def update(self, logits: Tensor, **batch: Any) -> None:
        per_token = logits.detach().double()
        labels = batch["label"].detach().to(torch.int64)
        token_bytes = batch["token_bytes"].detach().to(labels.device)
        if per_token.shape != labels.shape:
            raise ValueError(f"per-token loss has shape {tuple(per_token.shape)} but the targets have {tuple(labels.shape)}.")
        valid = int(batch.get("valid_count", labels.shape[0]))
        if not 0 <= valid <= labels.shape[0]:
            raise ValueError(f"valid_count {valid} is outside the batch's {labels.shape[0]} rows.")
        per_token, labels = per_token[:valid], labels[:valid]
        lengths = token_bytes[labels.reshape(-1)]
        counted = lengths > 0
        self.nats += float(per_token.reshape(-1)[counted].sum())
        self.bytes += int(lengths[counted].sum())

    def compute(self) -> dict[str, float]:
        t = _reduce(torch.tensor([self.nats, float(self.bytes)], dtype=torch.float64))
        if t[1] <= 0:
            raise ValueError("bits per byte scored no tokens: the eval produced no batches.")
        return {"bpb": float(t[0] / (math.log(2) * t[1]))}

    def state_dict(self) -> dict[str, Any]:
        return {"nats": self.nats, "bytes": self.bytes}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.nats, self.bytes = float(s["nats"]), int(s["bytes"])
