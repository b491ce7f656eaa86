"""Metric trackers (``priml/train/tracker.py:49-678``): JSON-lines file, TensorBoard,
W&B (rank 0, only when the package is importable), an async single-worker
wrapper and a fan-out list."""

from __future__ import annotations

import json
import queue
import threading
import time
from dataclasses import field
from pathlib import Path
from typing import Any

from priml_b200.config import Fig
from priml_b200.parallel.runtime import is_rank_zero

__all__ = ["AsyncTracker", "FileTracker", "NoTracker", "TensorBoardTracker", "TrackerList", "WandbTracker"]


def _scalar(v: Any) -> Any:
    try:
        return float(v)
    except (TypeError, ValueError):
        return str(v)


class NoTracker:
    class Config(Fig["NoTracker"]):
        pass

    def __init__(self, config: Any = None) -> None:
        del config

    def log(self, metrics: dict[str, Any], step: int) -> None:
        del metrics, step

    def flush(self) -> None:
        pass

    def close(self) -> None:
        pass


class FileTracker(NoTracker):
    """Appends ``{"step": s, "time": t, **metrics}`` lines to ``path`` (rank 0)."""

    class Config(Fig["FileTracker"]):
        path: str = "metrics.jsonl"

    def __init__(self, config: Config) -> None:
        self.path = Path(config.path)
        self._fh = None
        if is_rank_zero():
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self._fh = self.path.open("a")

    def log(self, metrics: dict[str, Any], step: int) -> None:
        if self._fh is None:
            return
        rec = {"step": step, "time": time.time(), **{k: _scalar(v) for k, v in metrics.items()}}
        self._fh.write(json.dumps(rec) + "\n")

    def flush(self) -> None:
        if self._fh is not None:
            self._fh.flush()

    def close(self) -> None:
        if self._fh is not None:
            self._fh.close()
            self._fh = None


class TensorBoardTracker(NoTracker):
    class Config(Fig["TensorBoardTracker"]):
        log_dir: str = "tensorboard"

    def __init__(self, config: Config) -> None:
        self.writer = None
        if is_rank_zero():
            try:
                from torch.utils.tensorboard import SummaryWriter

                self.writer = SummaryWriter(config.log_dir)
            except ImportError:
                self.writer = None

    def log(self, metrics: dict[str, Any], step: int) -> None:
        if self.writer is not None:
            for k, v in metrics.items():
                s = _scalar(v)
                if isinstance(s, float):
                    self.writer.add_scalar(k, s, step)

    def close(self) -> None:
        if self.writer is not None:
            self.writer.close()


class WandbTracker(NoTracker):
    class Config(Fig["WandbTracker"]):
        project: str = "priml_b200"
        name: str | None = None
        mode: str = "offline"

    def __init__(self, config: Config) -> None:
        self.run = None
        if is_rank_zero():
            try:
                import wandb  # type: ignore[import-not-found]

                self.run = wandb.init(project=config.project, name=config.name, mode=config.mode)
            except ImportError:
                self.run = None

    def log(self, metrics: dict[str, Any], step: int) -> None:
        if self.run is not None:
            self.run.log({k: _scalar(v) for k, v in metrics.items()}, step=step)

    def close(self) -> None:
        if self.run is not None:
            self.run.finish()


class AsyncTracker(NoTracker):
    """Runs another tracker's ``log`` on one worker thread."""

    class Config(Fig["AsyncTracker"]):
        inner: Any = field(default_factory=FileTracker.Config)

    def __init__(self, config: Config) -> None:
        self.inner = config.inner.make()
        self.q: queue.Queue = queue.Queue()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self) -> None:
        while True:
            item = self.q.get()
            if item is None:
                break
            self.inner.log(*item)
            self.q.task_done()

    def log(self, metrics: dict[str, Any], step: int) -> None:
        self.q.put((dict(metrics), step))

    def flush(self) -> None:
        self.q.join()
        self.inner.flush()

    def close(self) -> None:
        self.q.put(None)
        self.t.join(timeout=30)
        self.inner.close()


class TrackerList(NoTracker):
    class Config(Fig["TrackerList"]):
        trackers: list[Any] = field(default_factory=list)

    def __init__(self, config: Config) -> None:
        self.trackers = [t.make() for t in config.trackers]

    def log(self, metrics: dict[str, Any], step: int) -> None:
        for t in self.trackers:
            t.log(metrics, step)

    def flush(self) -> None:
        for t in self.trackers:
            t.flush()

    def close(self) -> None:
        for t in self.trackers:
            t.close()
