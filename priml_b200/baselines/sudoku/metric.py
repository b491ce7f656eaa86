"""Whole-grid and per-cell accuracy (``priml/baselines/sudoku/metric.py:1-120``).

``update(model_output, **batch)`` takes the eval step's packed output: the last
``grid_len`` columns are the decoded grid (any leading columns, such as the
halt logit, are ignored). Rows past ``valid_count`` are padding and skipped;
cells labelled ``ignore_label_id`` count neither way. ``compute()`` returns
``{"exact": solved / puzzles, "cell": right cells / cells}``, summed over ranks.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor

from priml_b200.config import Fig

__all__ = ["GridAccuracy", "all_reduce_counts"]


def all_reduce_counts(values: list[float]) -> list[float]:
    t = torch.tensor(values, dtype=torch.float64)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        if dist.get_backend() != "gloo":
            t = t.to(torch.device("cuda", torch.cuda.current_device()))
        dist.all_reduce(t)
    return t.cpu().tolist()


class GridAccuracy:
    class Config(Fig["GridAccuracy"]):
        ignore_label_id: int = -100

    def __init__(self, config: Config | None = None) -> None:
        self.config = config or GridAccuracy.Config()
        self.reset()

    def reset(self) -> None:
        self.solved = 0
        self.puzzles = 0
        self.cells_correct = 0
        self.cells = 0

    def update(self, logits: Tensor, **batch: Any) -> None:
        labels = batch["label"].detach().long()
        n = labels.shape[-1]
        pred = logits.detach()[:, -n:].long()
        labels = labels.to(pred.device)
        valid = int(batch.get("valid_count", labels.shape[0]))
        pred, labels = pred[:valid], labels[:valid]
        counted = labels != self.config.ignore_label_id
        right = (pred == labels) & counted
        per = counted.sum(-1)
        # one device -> host transfer for all four counts
        counts = torch.stack([((right.sum(-1) == per) & (per > 0)).sum(), (per > 0).sum(), right.sum(), per.sum()])
        s, p, cc, c = (int(v) for v in counts.cpu())
        self.solved += s
        self.puzzles += p
        self.cells_correct += cc
        self.cells += c

    def compute(self) -> dict[str, float]:
        solved, puzzles, cc, cells = all_reduce_counts([self.solved, self.puzzles, self.cells_correct, self.cells])
        return {"exact": solved / max(1.0, puzzles), "cell": cc / max(1.0, cells)}

    def state_dict(self) -> dict[str, Any]:
        return {"solved": self.solved, "puzzles": self.puzzles, "cells_correct": self.cells_correct, "cells": self.cells}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.solved = int(s.get("solved", 0))
        self.puzzles = int(s.get("puzzles", 0))
        self.cells_correct = int(s.get("cells_correct", 0))
        self.cells = int(s.get("cells", 0))
