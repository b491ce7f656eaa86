"""Checkpointable step timer (``priml/timer.py:24-105``): global (checkpointed)
and local (this process) counts and seconds; not re-entrant."""

from __future__ import annotations

import time
from typing import Any

__all__ = ["CheckpointableStepTimer"]


class CheckpointableStepTimer:
    def __init__(self) -> None:
        self.global_count = 0
        self.global_sec = 0.0
        self.local_count = 0
        self.local_sec = 0.0
        self._t0: float | None = None

    def __enter__(self) -> CheckpointableStepTimer:
        if self._t0 is not None:
            raise RuntimeError("CheckpointableStepTimer is not re-entrant")
        self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc: Any) -> None:
        assert self._t0 is not None
        dt = time.perf_counter() - self._t0
        self._t0 = None
        self.global_count += 1
        self.local_count += 1
        self.global_sec += dt
        self.local_sec += dt

    @property
    def mean_sec(self) -> float:
        return self.global_sec / self.global_count if self.global_count else 0.0

    def state_dict(self) -> dict[str, Any]:
        return {"global_count": self.global_count, "global_sec": self.global_sec}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        """Restore the checkpointed totals; this process's own counts start again at zero."""
        self.global_count = int(state.get("global_count", 0))
        self.global_sec = float(state.get("global_sec", 0.0))
        self.local_count = 0
        self.local_sec = 0.0
