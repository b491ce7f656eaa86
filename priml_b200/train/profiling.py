"""Profiling (``priml/train/profiling.py:31-752``).

* ``TorchProfiling``: a ``torch.profiler`` window over selected steps/ranks with
  Chrome-trace export and an optional CUDA memory snapshot.
* ``PhaseTimer``: named nested phases with inclusive/self wall time, plus
  ``measure_cuda`` CUDA-event pairs resolved lazily (no hot-path sync), and a
  rank-0 heartbeat thread that logs the current phase while a phase is open.
* ``nvtx_range``: NVTX ranges for external timeline tools.
"""

from __future__ import annotations

import contextlib
import logging
import threading
import time
from collections import defaultdict
from collections.abc import Iterator
from dataclasses import field
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from priml_b200.config import Fig

__all__ = ["PhaseTimer", "TorchProfiling", "nvtx_range"]

log = logging.getLogger(__name__)


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class TorchProfiling:
    class Config(Fig["TorchProfiling"]):
        torch_profile_start: int = 10
        torch_profile_end: int = 12
        ranks: list[int] = field(default_factory=lambda: [0])
        profile_cuda: bool = True
        output_dir: str = "profiles_out"
        memory_snapshot: bool = False

    def __init__(self, config: Config) -> None:
        self.config = config
        self.prof: Any = None
        rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
        self.enabled = rank in config.ranks
        self.rank = rank

    def on_step_start(self, step: int) -> None:
        if not self.enabled or step != self.config.torch_profile_start:
            return
        acts = [torch.profiler.ProfilerActivity.CPU]
        if self.config.profile_cuda and torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        if self.config.memory_snapshot and torch.cuda.is_available():
            torch.cuda.memory._record_memory_history()  # noqa: SLF001
        self.prof = torch.profiler.profile(activities=acts, record_shapes=False)
        self.prof.__enter__()

    def on_step_end(self, step: int) -> None:
        if self.prof is None or step != self.config.torch_profile_end:
            return
        self.prof.__exit__(None, None, None)
        out = Path(self.config.output_dir)
        out.mkdir(parents=True, exist_ok=True)
        self.prof.export_chrome_trace(str(out / f"trace_step_{step}_rank{self.rank}.json.gz"))
        log.info("top ops:\n%s", self.prof.key_averages().table(sort_by="self_cuda_time_total", row_limit=15))
        if self.config.memory_snapshot and torch.cuda.is_available():
            torch.cuda.memory._dump_snapshot(str(out / f"memory_step_{step}.pickle"))  # noqa: SLF001
            torch.cuda.memory._record_memory_history(enabled=None)  # noqa: SLF001
        self.prof = None


class PhaseTimer:
    class Config(Fig["PhaseTimer"]):
        heartbeat_sec: float = 0.0

    def __init__(self, config: Config | None = None) -> None:
        self.config = config or PhaseTimer.Config()
        self.total: dict[str, float] = defaultdict(float)
        self.child: dict[str, float] = defaultdict(float)
        self.count: dict[str, int] = defaultdict(int)
        self.stack: list[tuple[str, float]] = []
        self.cuda_pending: list[tuple[str, Any, Any]] = []
        self.cuda_ms: dict[str, float] = defaultdict(float)
        self._hb: threading.Thread | None = None
        self._stop = threading.Event()
        if self.config.heartbeat_sec > 0:
            self._hb = threading.Thread(target=self._heartbeat, daemon=True)
            self._hb.start()

    def _heartbeat(self) -> None:
        while not self._stop.wait(self.config.heartbeat_sec):
            if self.stack:
                name, t0 = self.stack[-1]
                log.info("heartbeat: in phase %s for %.1fs", name, time.perf_counter() - t0)

    @contextlib.contextmanager
    def phase(self, name: str) -> Iterator[None]:
        full = "/".join([s[0] for s in self.stack] + [name])
        t0 = time.perf_counter()
        self.stack.append((full, t0))
        try:
            with nvtx_range(name):
                yield
        finally:
            self.stack.pop()
            dt = time.perf_counter() - t0
            self.total[full] += dt
            self.count[full] += 1
            if self.stack:
                self.child[self.stack[-1][0]] += dt

    @contextlib.contextmanager
    def measure_cuda(self, name: str) -> Iterator[None]:
        if not torch.cuda.is_available():
            yield
            return
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        try:
            yield
        finally:
            e.record()
            self.cuda_pending.append((name, s, e))

    def resolve(self) -> None:
        keep = []
        for name, s, e in self.cuda_pending:
            if e.query():
                self.cuda_ms[name] += s.elapsed_time(e)
            else:
                keep.append((name, s, e))
        self.cuda_pending = keep

    def summary(self) -> dict[str, float]:
        self.resolve()
        out = {f"timing/{k}": v for k, v in self.total.items()}
        out.update({f"timing/{k}_self": v - self.child.get(k, 0.0) for k, v in self.total.items()})
        out.update({f"timing/cuda/{k}_ms": v for k, v in self.cuda_ms.items()})
        return out

    def close(self) -> None:
        self._stop.set()
