"""Sudoku puzzles served from device memory (``priml/baselines/sudoku/data.py:1-403``).

On-disk format (one directory per split, written by
:mod:`priml_b200.baselines.sudoku.prepare_data`): ``all__inputs.npy`` and
``all__labels.npy`` (``[rows, 81]`` ints; 1 = blank, 2..10 = digits 1..9),
``all__group_indices.npy`` (``[puzzles + 1]`` row bounds: each puzzle's
transformed copies are contiguous) and ``dataset.json`` (``vocab_size``).

Both splits are loaded onto the device once; an epoch shuffles rows within
each puzzle, then the whole order, and slices batches by index -- no host
transfer per step. Training batches get a fresh digit relabeling and one of
the eight square symmetries per row (:func:`augment_sudoku`), drawn on device.
The last short batch is zero-padded and reports ``valid_count``.
"""

from __future__ import annotations

import functools
import json
import logging
import math
from collections.abc import Iterator
from pathlib import Path
from typing import Any

import numpy as np
import torch
from torch import Tensor

from priml_b200.config import Fig
from priml_b200.parallel.runtime import get_device
from priml_b200.paths import resolve_working_dir
from priml_b200.timer import CheckpointableStepTimer

__all__ = ["SudokuData", "augment_sudoku", "load_split"]

log = logging.getLogger(__name__)


@functools.cache
def _square_symmetries(n: int, device: torch.device) -> Tensor:
    """``[8, n*n]`` gather indices of the dihedral group of the square (rotations, each with a mirror)."""
    base = torch.arange(n * n, device=device).view(n, n)
    out = []
    for k in range(4):
        r = torch.rot90(base, k)
        out += [r.reshape(-1), r.flip(1).reshape(-1)]
    return torch.stack(out)


def augment_sudoku(inputs: Tensor, labels: Tensor, *, vocab_size: int = 11,
                   generator: torch.Generator | None = None) -> tuple[Tensor, Tensor]:  # fmt: skip
    """Per row: a random relabeling of digit tokens 2..10 and a random square symmetry.

    Both preserve validity: a relabeled or rotated/mirrored solution still
    satisfies every row, column and box constraint.
    """
    b, dev = inputs.shape[0], inputs.device
    perm = torch.arange(vocab_size, device=dev).expand(b, -1).clone()
    perm[:, 2:11] = torch.rand(b, 9, device=dev, generator=generator).argsort(dim=1) + 2
    inputs = perm.gather(1, inputs.long()).to(inputs.dtype)
    labels = perm.gather(1, labels.long()).to(labels.dtype)
    sym = _square_symmetries(9, dev)[torch.randint(0, 8, (b,), device=dev, generator=generator)]
    return inputs.gather(1, sym), labels.gather(1, sym)


def load_split(dataset_dir: Path | str, split: str) -> dict[str, Any]:
    path = Path(dataset_dir).expanduser() / split
    meta = path / "dataset.json"
    if not meta.is_file():
        raise FileNotFoundError(
            f"no prepared sudoku data at {path}; build it with `python -m priml_b200.baselines.sudoku.prepare_data`."
        )
    info = json.loads(meta.read_text())
    return {
        "inputs": torch.from_numpy(np.load(path / "all__inputs.npy")).to(torch.int32),
        "labels": torch.from_numpy(np.load(path / "all__labels.npy")).to(torch.int32),
        "group_indices": torch.from_numpy(np.load(path / "all__group_indices.npy")).long(),
        "vocab_size": int(info["vocab_size"]),
    }


class _Batches:
    def __init__(self, *, dataset_dir: Path, device: Any, batch_size: int, split: str, shuffle: bool,
                 num_puzzles: int | None, seed: int | None, epoch: int, augment: bool,
                 augment_seed: int | None) -> None:  # fmt: skip
        if epoch < 0:
            raise ValueError(f"epoch must be non-negative; got {epoch}.")
        data = load_split(dataset_dir, split)
        bounds = data["group_indices"]
        if num_puzzles is not None and num_puzzles < len(bounds) - 1:
            bounds = bounds[: num_puzzles + 1]
        rows = int(bounds[-1])
        self.device = get_device(device)
        self.inputs = data["inputs"][:rows].to(self.device)
        self.labels = data["labels"][:rows].to(self.device)
        self.bounds = bounds
        self.vocab_size = data["vocab_size"]
        self.batch_size = batch_size
        self.shuffle = shuffle
        self.seed = seed
        self.augment = augment
        self.epoch = epoch
        self._augment_gen: torch.Generator | None = None
        if augment and augment_seed is not None:
            self._augment_gen = torch.Generator(device=self.device)
            self._augment_gen.manual_seed(augment_seed)
        # puzzle id of every row, so the within-puzzle shuffle is one sort on device
        sizes = (bounds[1:] - bounds[:-1]).to(self.device)
        self._group = torch.repeat_interleave(torch.arange(len(sizes), device=self.device), sizes)

    def _order(self) -> Tensor:
        n = int(self.bounds[-1])
        if not self.shuffle:
            return torch.arange(n, device=self.device)
        gen = None
        if self.seed is not None:
            gen = torch.Generator(device=self.device)
            gen.manual_seed(self.seed + self.epoch)
        # within-puzzle shuffle: sort by (puzzle, random key); then shuffle the whole order
        key = torch.rand(n, device=self.device, generator=gen, dtype=torch.float64) + self._group.double()
        within = key.argsort()
        return within[torch.randperm(n, device=self.device, generator=gen)]

    def __iter__(self) -> Iterator[dict[str, Any]]:
        order = self._order()
        self.epoch += 1
        bs = self.batch_size
        for start in range(0, order.numel(), bs):
            idx = order[start : start + bs]
            valid = idx.numel()
            inputs, labels = self.inputs[idx], self.labels[idx]
            if valid < bs:
                pad = bs - valid
                inputs = torch.cat([inputs, inputs.new_zeros(pad, inputs.shape[1])])
                labels = torch.cat([labels, labels.new_zeros(pad, labels.shape[1])])
            if self.augment:
                inputs, labels = augment_sudoku(inputs, labels, vocab_size=self.vocab_size, generator=self._augment_gen)
            yield {"media": inputs, "label": labels, "valid_count": valid}

    def __len__(self) -> int:
        return math.ceil(int(self.bounds[-1]) / self.batch_size)


class SudokuData:
    class Config(Fig["SudokuData"]):
        base_dir: Path | str | None = None
        working_dir: Path | str = "/datasets/sudoku-extreme"
        batch_size: int = 384
        eval_batch_size: int | None = None
        device: str = "auto"
        augment: bool = True
        seed: int | None = None
        """Shuffle seed; an int seeds epoch ``e`` with ``seed + e``."""
        augment_seed: int | None = None
        num_train_puzzles: int | None = None
        num_eval_puzzles: int | None = None

        def finalize(self):  # noqa: ANN201
            self.working_dir = resolve_working_dir(self.working_dir, self.base_dir)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        self.config = config
        self.dataset_dir = Path(config.working_dir)
        self.batch_size = config.batch_size
        self.eval_batch_size = config.eval_batch_size or config.batch_size
        self.timer_epoch = CheckpointableStepTimer()
        self._epochs = 0
        self._live: _Batches | None = None

    def train_dataloader(self) -> _Batches:
        if self._live is not None:
            self._epochs = self._live.epoch
        c = self.config
        self._live = _Batches(dataset_dir=self.dataset_dir, device=c.device, batch_size=self.batch_size, split="train",
                              shuffle=True, num_puzzles=c.num_train_puzzles, seed=c.seed, epoch=self._epochs,
                              augment=c.augment, augment_seed=c.augment_seed)  # fmt: skip
        return self._live

    def eval_dataloader(self) -> _Batches:
        c = self.config
        return _Batches(dataset_dir=self.dataset_dir, device=c.device, batch_size=self.eval_batch_size, split="test",
                        shuffle=False, num_puzzles=c.num_eval_puzzles, seed=c.seed, epoch=0, augment=False,
                        augment_seed=None)  # fmt: skip

    def state_dict(self) -> dict[str, Any]:
        return {"timer_epoch": self.timer_epoch.state_dict()}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        if "timer_epoch" in s:
            self.timer_epoch.load_state_dict(s["timer_epoch"])
            self._epochs = self.timer_epoch.global_count
            if self._live is not None:
                self._live.epoch = self._epochs
