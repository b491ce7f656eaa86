"""Logging setup (``priml/logger.py:25-219``): a compact formatter with rank and
elapsed time, and a replay buffer so lines logged before stdout was rebound
(e.g. inside a launcher) can be re-emitted."""

from __future__ import annotations

import logging
import os
import sys
import time
from typing import TextIO

__all__ = ["Timer", "bind_logging_to_current_stdout", "replay_buffered_logs", "setup_logging"]

_T0 = time.time()


class Timer:
    """``with Timer() as t: ...; t.elapsed`` (seconds)."""

    def __enter__(self) -> Timer:
        self.start = time.perf_counter()
        self.elapsed = 0.0
        return self

    def __exit__(self, *exc: object) -> None:
        self.elapsed = time.perf_counter() - self.start


class CustomFormatter(logging.Formatter):
    def format(self, record: logging.LogRecord) -> str:
        rank = os.environ.get("RANK", "0")
        el = record.created - _T0
        return f"[{el:8.1f}s r{rank} {record.levelname[0]} {record.name.rsplit('.', 1)[-1]}] {record.getMessage()}"


class _Replay(logging.Handler):
    def __init__(self, capacity: int = 1000) -> None:
        super().__init__()
        self.records: list[logging.LogRecord] = []
        self.capacity = capacity

    def emit(self, record: logging.LogRecord) -> None:
        self.records.append(record)
        if len(self.records) > self.capacity:
            self.records.pop(0)


_replay = _Replay()


class _Stdout(logging.StreamHandler):
    def __init__(self, stream: TextIO | None = None) -> None:
        super().__init__(stream or sys.stdout)


def setup_logging(level: str = "INFO") -> None:
    root = logging.getLogger()
    root.setLevel(getattr(logging, level.upper(), logging.INFO))
    for h in list(root.handlers):
        if isinstance(h, (_Stdout, _Replay)):
            root.removeHandler(h)
    h = _Stdout()
    h.setFormatter(CustomFormatter())
    root.addHandler(h)
    root.addHandler(_replay)


def bind_logging_to_current_stdout() -> None:
    for h in logging.getLogger().handlers:
        if isinstance(h, _Stdout):
            h.setStream(sys.stdout)


def replay_buffered_logs() -> None:
    fmt = CustomFormatter()
    for r in _replay.records:
        sys.stdout.write(fmt.format(r) + "\n")
