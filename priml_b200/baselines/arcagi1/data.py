"""ARC-AGI tasks served from device memory (``priml/baselines/arcagi1/data.py:1-363``).

On-disk layout (one directory per split): ``all__inputs.npy`` / ``all__labels.npy``
(``[rows, 900]`` ints: 0 = pad, 1 = end-of-grid marker, 2..11 = the ten colors),
``all__puzzle_indices.npy`` (``[puzzles + 1]`` row bounds: one puzzle is one
augmented view of a task), ``all__group_indices.npy`` (``[tasks + 1]`` puzzle
bounds), ``all__puzzle_identifiers.npy`` (``[puzzles]`` rows of the per-puzzle
embedding table) and ``dataset.json`` (``vocab_size``, ``ignore_label_id``).

Training samples hierarchically so every TASK weighs the same: a seeded
permutation of tasks; for each task one random view; from it as many of its
example rows (without replacement) as still fit the batch. Batches are always
full -- the tail that cannot fill one is dropped. Evaluation walks every row in
order, pads the last batch and reports ``valid_count``. Labels equal to the
pad id become ``-100`` so the loss and metrics skip them.
"""

from __future__ import annotations

import json
import logging
import math
from collections.abc import Iterator
from pathlib import Path
from typing import Any

import numpy as np
import torch

from priml_b200.config import Fig
from priml_b200.parallel.runtime import get_device
from priml_b200.paths import resolve_working_dir
from priml_b200.timer import CheckpointableStepTimer

__all__ = ["ArcData", "load_split", "num_puzzle_identifiers"]

log = logging.getLogger(__name__)

IGNORE = -100


def load_split(dataset_dir: Path | str, split: str) -> dict[str, Any]:
    path = Path(dataset_dir).expanduser() / split
    meta = path / "dataset.json"
    if not meta.is_file():
        raise FileNotFoundError(
            f"no prepared ARC data at {path}; build it with `python -m priml_b200.baselines.arcagi1.prepare_data`."
        )
    info = json.loads(meta.read_text())
    return {
        "inputs": torch.from_numpy(np.load(path / "all__inputs.npy")).to(torch.int32),
        "labels": torch.from_numpy(np.load(path / "all__labels.npy")).to(torch.int32),
        "puzzle_indices": np.load(path / "all__puzzle_indices.npy").astype(np.int64),
        "group_indices": np.load(path / "all__group_indices.npy").astype(np.int64),
        "puzzle_identifiers": np.load(path / "all__puzzle_identifiers.npy").astype(np.int64),
        "ignore_label_id": int(info.get("ignore_label_id", 0)),
    }


def num_puzzle_identifiers(dataset_dir: Path | str) -> int:
    """Rows the per-puzzle table needs: ``dataset.json``'s count, else one past the largest identifier."""
    root = Path(dataset_dir).expanduser()
    meta = root / "train" / "dataset.json"
    if not meta.is_file():
        raise FileNotFoundError(f"no prepared ARC data at {root}; the per-puzzle table cannot be sized.")
    info = json.loads(meta.read_text())
    if "num_puzzle_identifiers" in info:
        return int(info["num_puzzle_identifiers"])
    top = [int(np.load(root / s / "all__puzzle_identifiers.npy").max(initial=0)) for s in ("train", "test")
           if (root / s / "all__puzzle_identifiers.npy").is_file()]  # fmt: skip
    return max(top) + 1


class _Batches:
    def __init__(self, *, dataset_dir: Path, device: Any, batch_size: int, split: str, sample_by_task: bool,
                 num_tasks: int | None, seed: int, passes: int) -> None:  # fmt: skip
        d = load_split(dataset_dir, split)
        groups, puzzles = d["group_indices"], d["puzzle_indices"]
        if num_tasks is not None and num_tasks < len(groups) - 1:
            groups = groups[: num_tasks + 1]
            puzzles = puzzles[: int(groups[-1]) + 1]
        rows = int(puzzles[-1])
        self.device = get_device(device)
        self.inputs = d["inputs"][:rows].to(self.device)
        labels = d["labels"][:rows]
        self.labels = labels.masked_fill(labels == d["ignore_label_id"], IGNORE).to(self.device)
        self.groups, self.puzzles = groups, puzzles
        self.identifiers = d["puzzle_identifiers"][: len(puzzles) - 1]
        self.batch_size = batch_size
        self.sample_by_task = sample_by_task
        self.seed = seed
        self.passes = passes

    @property
    def num_tasks(self) -> int:
        return len(self.groups) - 1

    def __len__(self) -> int:
        return math.ceil(int(self.puzzles[-1]) / self.batch_size)

    def __iter__(self) -> Iterator[dict[str, Any]]:
        return self._sampled() if self.sample_by_task else self._ordered()

    def _sampled(self) -> Iterator[dict[str, Any]]:
        rng = np.random.Generator(np.random.Philox(seed=self.seed + self.passes))
        self.passes += 1
        order = rng.permutation(self.num_tasks)
        bs, cursor = self.batch_size, 0
        while cursor < order.size:
            rows, ids, filled = [], [], 0
            while cursor < order.size and filled < bs:
                task = int(order[cursor])
                cursor += 1
                lo, hi = int(self.groups[task]), int(self.groups[task + 1])
                if hi <= lo:
                    continue
                view = int(rng.integers(lo, hi))
                start, size = int(self.puzzles[view]), int(self.puzzles[view + 1] - self.puzzles[view])
                take = min(size, bs - filled)
                rows.append(start + rng.choice(size, take, replace=False))
                ids.append(np.full(take, view, dtype=np.int64))
                filled += take
            if filled < bs:
                return
            yield self._batch(np.concatenate(rows), np.concatenate(ids), bs)

    def _ordered(self) -> Iterator[dict[str, Any]]:
        total = int(self.puzzles[-1])
        for start in range(0, total, self.batch_size):
            rows = np.arange(start, min(total, start + self.batch_size), dtype=np.int64)
            views = np.searchsorted(self.puzzles, rows, side="right") - 1
            yield self._batch(rows, views, rows.size)

    def _batch(self, rows: np.ndarray, views: np.ndarray, valid: int) -> dict[str, Any]:
        idx = torch.from_numpy(rows.astype(np.int64)).to(self.device)
        media, labels = self.inputs[idx], self.labels[idx]
        ids = torch.from_numpy(self.identifiers[views]).to(self.device)
        pad = self.batch_size - valid
        if pad:
            media = torch.cat([media, media.new_zeros(pad, media.shape[1])])
            labels = torch.cat([labels, labels.new_full((pad, labels.shape[1]), IGNORE)])
            ids = torch.cat([ids, ids.new_zeros(pad)])
        return {"media": media, "label": labels, "valid_count": valid, "puzzle_identifiers": ids}


class ArcData:
    class Config(Fig["ArcData"]):
        base_dir: Path | str | None = None
        working_dir: Path | str = "/datasets/arcagi1"
        batch_size: int = 256
        eval_batch_size: int | None = None
        device: str = "auto"
        seed: int = 0
        num_tasks: int | None = None
        num_eval_tasks: int | None = None

        def finalize(self):  # noqa: ANN201
            self.working_dir = resolve_working_dir(self.working_dir, self.base_dir)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        self.config = config
        self.dataset_dir = Path(config.working_dir)
        self.batch_size = config.batch_size
        self.eval_batch_size = config.eval_batch_size or config.batch_size
        self.timer_epoch = CheckpointableStepTimer()
        self._passes = 0
        self._live: _Batches | None = None

    def train_dataloader(self) -> _Batches:
        if self._live is not None:
            self._passes = self._live.passes
        c = self.config
        self._live = _Batches(dataset_dir=self.dataset_dir, device=c.device, batch_size=self.batch_size, split="train",
                              sample_by_task=True, num_tasks=c.num_tasks, seed=c.seed, passes=self._passes)  # fmt: skip
        return self._live

    def eval_dataloader(self) -> _Batches:
        c = self.config
        return _Batches(dataset_dir=self.dataset_dir, device=c.device, batch_size=self.eval_batch_size, split="test",
                        sample_by_task=False, num_tasks=c.num_eval_tasks, seed=c.seed, passes=0)  # fmt: skip

    def state_dict(self) -> dict[str, Any]:
        return {"passes": self._live.passes if self._live is not None else self._passes,
                "timer_epoch": self.timer_epoch.state_dict()}  # fmt: skip

    def load_state_dict(self, s: dict[str, Any]) -> None:
        if "passes" in s:
            self._passes = int(s["passes"])
            if self._live is not None:
                self._live.passes = self._passes
        if "timer_epoch" in s:
            self.timer_epoch.load_state_dict(s["timer_epoch"])
