"""pass@K over ranked answers per puzzle (``priml/baselines/arcagi1/metric.py:1-153``).

``update(packed, **batch)`` reads the eval step's packed rows (column 0 the
halt logit, the last ``grid_len`` columns the decoded grid) with the batch's
``label`` and ``puzzle_identifiers``. Each valid row casts one vote for its
answer (the grid's counted cells, hashed) under its puzzle. ``compute()`` ranks
each puzzle's answers by vote count, ties broken by mean halt confidence
(``sigmoid`` of the halt logit), and reports the fraction of puzzles whose true
grid is among the top K for every configured K, summed over ranks.
"""

from __future__ import annotations

import hashlib
from typing import Any

import torch
from torch import Tensor

from priml_b200.baselines.sudoku.metric import all_reduce_counts
from priml_b200.config import Fig

__all__ = ["PassK"]


def _digest(cells: Tensor) -> str:
    return hashlib.blake2b(cells.to(torch.int16).cpu().numpy().tobytes(), digest_size=16).hexdigest()


class PassK:
    class Config(Fig["PassK"]):
        pass_ks: tuple[int, ...] = (1, 2, 5, 10)
        ignore_label_id: int = -100

    def __init__(self, config: Config | None = None) -> None:
        self.config = config or PassK.Config()
        self.reset()

    def reset(self) -> None:
        self._votes: dict[int, dict[str, list[float]]] = {}
        self._truth: dict[int, str] = {}

    def update(self, logits: Tensor, **batch: Any) -> None:
        labels = batch["label"].detach().long()
        n = labels.shape[-1]
        packed = logits.detach()
        valid = int(batch.get("valid_count", labels.shape[0]))
        pred = packed[:valid, -n:].long().cpu()
        conf = torch.sigmoid(packed[:valid, 0].float()).cpu()
        labels = labels[:valid].cpu()
        ids = batch["puzzle_identifiers"].detach()[:valid].long().cpu()
        counted = labels != self.config.ignore_label_id
        for r in range(pred.shape[0]):
            keep = counted[r]
            if not bool(keep.any()):
                continue
            puzzle = int(ids[r])
            self._truth.setdefault(puzzle, _digest(labels[r][keep]))
            tally = self._votes.setdefault(puzzle, {}).setdefault(_digest(pred[r][keep]), [0.0, 0.0])
            tally[0] += 1.0
            tally[1] += float(conf[r])

    def compute(self) -> dict[str, float]:
        ks = self.config.pass_ks
        hits = dict.fromkeys(ks, 0)
        for puzzle, tally in self._votes.items():
            ranked = sorted(tally.items(), key=lambda kv: (kv[1][0], kv[1][1] / kv[1][0]), reverse=True)
            answers = [a for a, _ in ranked]
            for k in ks:
                hits[k] += int(self._truth[puzzle] in answers[:k])
        total, *found = all_reduce_counts([float(len(self._votes)), *(float(hits[k]) for k in ks)])
        return {f"pass@{k}": h / max(1.0, total) for k, h in zip(ks, found, strict=True)}

    def state_dict(self) -> dict[str, Any]:
        return {"votes": self._votes, "truth": self._truth}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self._votes = s.get("votes", {})
        self._truth = s.get("truth", {})
