"""The dataset seam for an environment that generates its own data (``priml/baselines/craftax/data.py``).

The train loop iterates ``updates_per_epoch`` empty batches (each one update of
the learner, which collects its own rollout); evaluation batches carry the
learner's policy so that :class:`CraftaxScore` can play it.
"""

from __future__ import annotations

from collections.abc import Iterator
from typing import Any

from priml_b200.config import Fig
from priml_b200.timer import CheckpointableStepTimer

__all__ = ["CraftaxRollouts"]


class CraftaxRollouts:
    class Config(Fig["CraftaxRollouts"]):
        updates_per_epoch: int = 1000
        eval_batches: int = 1

    def __init__(self, config: Config | None = None) -> None:
        self.config = config or CraftaxRollouts.Config()
        if self.config.updates_per_epoch <= 0 or self.config.eval_batches <= 0:
            raise ValueError("rollout cadence must be positive")
        self.timer_epoch = CheckpointableStepTimer()
        self._step: Any = None

    def bind_step(self, step: Any) -> None:
        self._step = step

    def train_dataloader(self) -> Iterator[dict[str, Any]]:
        return iter([{"valid_count": 1} for _ in range(self.config.updates_per_epoch)])

    def eval_dataloader(self) -> Iterator[dict[str, Any]]:
        batch: dict[str, Any] = {"valid_count": 1}
        if self._step is not None:
            batch["policy"] = self._step.model
        return iter([dict(batch) for _ in range(self.config.eval_batches)])

    def state_dict(self) -> dict[str, Any]:
        return {"timer_epoch": self.timer_epoch.state_dict()}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        if "timer_epoch" in s:
            self.timer_epoch.load_state_dict(s["timer_epoch"])
