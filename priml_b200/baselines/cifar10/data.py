"""CIFAR-10 tensors served from device memory (``priml/baselines/cifar10/data.py:40-264``).

``prepare(directory)`` writes normalized ``train.pt`` / ``test.pt``
(``{"media": float [N, 3, 32, 32], "label": int64 [N]}``); ``Cifar10Data``
loads both splits onto the device once (channels-last) and slices shuffled
batches from them, so an epoch involves no host transfer at all.
"""

from __future__ import annotations

import logging
from collections.abc import Iterator, Sequence
from pathlib import Path
from typing import Any

import torch
from torch import Tensor

from priml_b200.config import Fig
from priml_b200.parallel.runtime import get_device

__all__ = ["CIFAR10_MEAN", "CIFAR10_STD", "Cifar10Data", "prepare", "prepare_from_arrays"]

log = logging.getLogger(__name__)

CIFAR10_MEAN = (0.4914, 0.4822, 0.4465)
CIFAR10_STD = (0.2470, 0.2435, 0.2616)


def prepare_from_arrays(directory: Path | str, split: str, images: Tensor, labels: Tensor, *,
                        mean: Sequence[float] = CIFAR10_MEAN, std: Sequence[float] = CIFAR10_STD) -> Path:  # fmt: skip
    """Normalize uint8 ``[N, 32, 32, 3]`` (or ``[N, 3, 32, 32]``) images and write ``{split}.pt``."""
    destination = Path(directory)
    destination.mkdir(parents=True, exist_ok=True)
    media = torch.as_tensor(images)
    if media.shape[-1] == 3:
        media = media.moveaxis(-1, -3)
    media = media.float().div(255)
    media = (media - torch.tensor(mean).view(1, 3, 1, 1)) / torch.tensor(std).view(1, 3, 1, 1)
    path = destination / f"{split}.pt"
    staging = path.with_suffix(".pt.partial")
    torch.save({"media": media.contiguous(), "label": torch.as_tensor(labels).long()}, staging)
    staging.replace(path)
    return path


def prepare(directory: Path | str) -> None:
    """Download CIFAR-10 (torchvision) and cache normalized splits; a present split is left alone."""
    destination = Path(directory)
    for split, train in (("train", True), ("test", False)):
        if (destination / f"{split}.pt").exists():
            continue
        import torchvision.datasets  # only needed where a split is missing

        source = torchvision.datasets.CIFAR10(str(destination), train=train, download=True)
        prepare_from_arrays(destination, split, torch.as_tensor(source.data), torch.as_tensor(source.targets))
        log.info("cifar10: wrote %s", split)


def _load_split(path: Path, device: torch.device, dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    if not path.is_file():
        raise FileNotFoundError(f"prepared CIFAR-10 split not found at {path}; run the baseline's prepare() first.")
    payload = torch.load(path, map_location="cpu", weights_only=True)
    missing = {"media", "label"} - set(payload)
    if missing:
        raise ValueError(f"{path} is not a prepared CIFAR-10 split: missing {sorted(missing)}.")
    media = payload["media"].to(device=device, dtype=dtype).contiguous(memory_format=torch.channels_last)
    return media, payload["label"].to(device)


class _BatchIterator:
    def __init__(self, media: Tensor, label: Tensor, *, batch_size: int, shuffle: bool, drop_last: bool) -> None:
        self.media, self.label = media, label
        self.batch_size, self.shuffle, self.drop_last = batch_size, shuffle, drop_last

    def __iter__(self) -> Iterator[dict[str, Tensor]]:
        n = len(self.media)
        order = torch.randperm(n, device=self.media.device) if self.shuffle else torch.arange(n, device=self.media.device)
        for start in range(0, n, self.batch_size):
            index = order[start : start + self.batch_size]
            if self.drop_last and len(index) < self.batch_size:
                return
            yield {"media": self.media[index], "label": self.label[index]}

    def __len__(self) -> int:
        n = len(self.media)
        return n // self.batch_size if self.drop_last else (n + self.batch_size - 1) // self.batch_size


class Cifar10Data:
    class Config(Fig["Cifar10Data"]):
        working_dir: str = "/datasets/cifar10"
        batch_size: int = 512
        eval_batch_size: int = 1000
        drop_last: bool = False
        device: str = "auto"
        dtype: torch.dtype = torch.float32

    def __init__(self, config: Config | None = None) -> None:
        config = config or Cifar10Data.Config()
        self.config = config
        self.device = get_device(config.device)
        root = Path(config.working_dir)
        self.train_media, self.train_label = _load_split(root / "train.pt", self.device, config.dtype)
        self.test_media, self.test_label = _load_split(root / "test.pt", self.device, config.dtype)

    def train_dataloader(self) -> _BatchIterator:
        return _BatchIterator(self.train_media, self.train_label, batch_size=self.config.batch_size, shuffle=True,
                              drop_last=self.config.drop_last)  # fmt: skip

    def eval_dataloader(self) -> _BatchIterator:
        return _BatchIterator(self.test_media, self.test_label, batch_size=self.config.eval_batch_size, shuffle=False,
                              drop_last=False)  # fmt: skip

    def state_dict(self) -> dict[str, Any]:
        return {}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        del state_dict
