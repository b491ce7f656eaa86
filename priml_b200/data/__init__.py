"""Datasets (``priml/data/``): the protocol, the seeded dummy dataset and a
synthetic token stream for language-model training."""

from __future__ import annotations

from collections.abc import Iterator
from typing import Any, Protocol

import torch
from torch import Tensor

from priml_b200.timer import CheckpointableStepTimer
from priml_b200.config import Fig

__all__ = ["DatasetProtocol", "DummyDataset", "SyntheticTokens"]


class DatasetProtocol(Protocol):
    def train_dataloader(self) -> Any: ...

    def eval_dataloader(self) -> Any: ...

    def state_dict(self) -> dict[str, Any]: ...

    def load_state_dict(self, state_dict: dict[str, Any]) -> None: ...


class DummyDataset:
    """Seeded random ``media`` / ``label`` batches (``priml/data/dummy.py:17-115``)."""

    class Config(Fig["DummyDataset"]):
        num_samples: int = 100
        batch_size: int = 32
        input_shape: tuple[int, ...] = (3, 224, 224)
        num_classes: int = 1000
        device: str | None = "cpu"
        seed: int = 0
        num_workers: int = 0

    def __init__(self, config: Config) -> None:
        self.config = config
        g = torch.Generator().manual_seed(config.seed)
        self.media = torch.randn((config.num_samples, *config.input_shape), generator=g)
        self.label = torch.randint(0, config.num_classes, (config.num_samples,), generator=g)
        self.timer_epoch = CheckpointableStepTimer()

    def _batches(self) -> Iterator[dict[str, Tensor]]:
        b = self.config.batch_size
        dev = self.config.device or "cpu"
        for i in range(0, self.config.num_samples - b + 1, b):
            yield {"media": self.media[i : i + b].to(dev), "label": self.label[i : i + b].to(dev)}

    def train_dataloader(self) -> Iterator[dict[str, Tensor]]:
        return self._batches()

    def eval_dataloader(self) -> Iterator[dict[str, Tensor]]:
        return self._batches()

    def state_dict(self) -> dict[str, Any]:
        return {"timer_epoch": self.timer_epoch.state_dict()}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        if "timer_epoch" in s:
            self.timer_epoch.load_state_dict(s["timer_epoch"])


class SyntheticTokens:
    """Uniform random tokens ``[batch, seq + 1]`` from a seeded generator, split
    into ``tokens`` / ``targets`` (targets = inputs shifted by one). Batches live
    in pinned host memory; :meth:`TrainStep.preprocess_batch` copies them to the
    device with ``non_blocking``. ``steps_per_epoch`` batches form an epoch."""

    class Config(Fig["SyntheticTokens"]):
        vocab_size: int = 32768
        batch_size: int = 4
        seq_len: int = 4096
        seed: int = 0
        steps_per_epoch: int = 1_000_000
        pin_memory: bool = True

    def __init__(self, config: Config) -> None:
        self.config = config
        self.timer_epoch = CheckpointableStepTimer()
        self._step = 0

    def _make(self, index: int) -> dict[str, Tensor]:
        c = self.config
        g = torch.Generator().manual_seed(c.seed * 1_000_003 + index)
        seq = torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len + 1), generator=g)
        batch = {"tokens": seq[:, :-1].contiguous(), "targets": seq[:, 1:].contiguous()}
        if c.pin_memory and torch.cuda.is_available():
            batch = {k: v.pin_memory() for k, v in batch.items()}
        return batch

    def train_dataloader(self) -> Iterator[dict[str, Tensor]]:
        while True:
            for _ in range(self.config.steps_per_epoch):
                yield self._make(self._step)
                self._step += 1
            return

    def eval_dataloader(self) -> Iterator[dict[str, Tensor]]:
        for i in range(4):
            yield self._make(-1 - i)

    def state_dict(self) -> dict[str, Any]:
        return {"step": self._step, "timer_epoch": self.timer_epoch.state_dict()}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self._step = int(s.get("step", 0))
        if "timer_epoch" in s:
            self.timer_epoch.load_state_dict(s["timer_epoch"])
from priml_b200.data import augmentation_gpu, environment  # noqa: E402, F401
