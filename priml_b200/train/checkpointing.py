"""Checkpoint save / resume (``priml/train/checkpointing.py:66-755``).

Format (kept compatible with the reference):

* file name ``step_{step:08d}.pt`` under ``working_dir``;
* states without DTensors: one ``torch.save`` file written by rank 0 to a
  temporary name and atomically renamed;
* states with DTensors (FSDP / TP): a DCP directory of the same name whose
  ``.metadata`` is written last -- a directory without it is incomplete and is
  skipped on resume (fallback past a crashed latest checkpoint);
* ``AsyncLocalStateDictStorer`` uses ``dcp.async_save`` and joins only at
  all-rank points (the next save, ``flush`` and ``load``).

Retention: ``keep_last_n`` newest plus every ``keep_every``-th step. The
overwrite guard refuses to start a run whose future saves would replace
checkpoints of a different (longer) run unless ``allow_checkpoint_overwrite``.
Rank-dependent decisions (does a checkpoint exist?) are agreed by broadcast.
"""

from __future__ import annotations

import logging
import os
import re
import shutil
from dataclasses import field
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from priml_b200.config import Fig
from priml_b200.parallel.runtime import is_rank_zero

__all__ = ["AsyncLocalStateDictStorer", "Checkpointer", "SyncLocalStateDictStorer"]

log = logging.getLogger(__name__)
_STEP_RE = re.compile(r"step_(\d+)")


def _dist() -> bool:
    return dist.is_available() and dist.is_initialized()


def _barrier() -> None:
    if _dist():
        dist.barrier()


def _has_dtensor(obj: Any) -> bool:
    from torch.distributed.tensor import DTensor

    if isinstance(obj, DTensor):
        return True
    if isinstance(obj, dict):
        return any(_has_dtensor(v) for v in obj.values())
    if isinstance(obj, (list, tuple)):
        return any(_has_dtensor(v) for v in obj)
    return False


def _agreed(value: Any) -> Any:
    """Rank 0's ``value`` on every rank."""
    if not _dist():
        return value
    box = [value]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def _is_complete(path: Path) -> bool:
    if path.is_dir():
        return (path / ".metadata").exists()
    return path.is_file()


class SyncLocalStateDictStorer:
    class Config(Fig["SyncLocalStateDictStorer"]):
        pass

    def __init__(self, config: Any = None) -> None:
        del config

    def write(self, path: Path, state: dict[str, Any], after_write: Any = None) -> None:
        if _has_dtensor(state):
            import torch.distributed.checkpoint as dcp

            dcp.save(state, checkpoint_id=str(path))
            _barrier()
        else:
            if is_rank_zero():
                tmp = path.with_name(path.name + ".tmp")
                torch.save(state, tmp)
                os.replace(tmp, path)
            _barrier()
        if after_write is not None and is_rank_zero():
            after_write()

    def read(self, path: Path, into: dict[str, Any]) -> dict[str, Any]:
        if path.is_dir():
            import torch.distributed.checkpoint as dcp

            dcp.load(into, checkpoint_id=str(path))
            return into
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
        state = torch.load(path, map_location=dev, weights_only=True)
        if "rng" in state:
            state["rng"] = _to_cpu(state["rng"])
        return state

    def flush(self) -> None:
        pass


def _to_cpu(x: Any) -> Any:
    if isinstance(x, torch.Tensor):
        return x.cpu()
    if isinstance(x, dict):
        return {k: _to_cpu(v) for k, v in x.items()}
    if isinstance(x, list):
        return [_to_cpu(v) for v in x]
    return x


class AsyncLocalStateDictStorer(SyncLocalStateDictStorer):
    """``dcp.async_save``; the pending future is joined at all-rank points only."""

    class Config(Fig["AsyncLocalStateDictStorer"]):
        pass

    def __init__(self, config: Any = None) -> None:
        super().__init__(config)
        self._pending: Any = None
        self._after: Any = None

    def write(self, path: Path, state: dict[str, Any], after_write: Any = None) -> None:
        import torch.distributed.checkpoint as dcp

        self.flush()
        if not _has_dtensor(state) and not _dist():
            super().write(path, state, after_write)
            return
        self._pending = dcp.async_save(state, checkpoint_id=str(path))
        self._after = after_write

    def flush(self) -> None:
        if self._pending is not None:
            self._pending.result()
            self._pending = None
            _barrier()
            if self._after is not None and is_rank_zero():
                self._after()
            self._after = None


class Checkpointer:
    class Config(Fig["Checkpointer"]):
        base_dir: Path | str | None = None
        working_dir: Path | str = "checkpoints"
        filename: str = "step_{step:08d}.pt"
        save_every: int = 1000
        keep_last_n: int = -1
        keep_every: int = 0
        storer: Any = field(default_factory=SyncLocalStateDictStorer.Config)
        resume: bool = True
        resume_step: int = -1
        allow_checkpoint_overwrite: bool = False

    def __init__(self, config: Config) -> None:
        self.config = config
        base = Path(config.base_dir) if config.base_dir is not None else Path(".")
        wd = Path(config.working_dir)
        self.dir = wd if wd.is_absolute() else base / wd
        self.storage = config.storer.make()
        if is_rank_zero():
            self.dir.mkdir(parents=True, exist_ok=True)
        _barrier()

    # ------------------------------------------------------------------ listing
    def path_for(self, step: int) -> Path:
        return self.dir / self.config.filename.format(step=step)

    def _list(self) -> list[tuple[int, Path]]:
        out = []
        if self.dir.exists():
            for p in self.dir.iterdir():
                m = _STEP_RE.match(p.name)
                if m and not p.name.endswith(".tmp") and _is_complete(p):
                    out.append((int(m.group(1)), p))
        return sorted(out)

    # ------------------------------------------------------------------ save
    def maybe_save(self, target: Any, step: int) -> bool:
        if self.config.save_every > 0 and step > 0 and step % self.config.save_every == 0:
            self.save(target, step)
            return True
        return False

    def save(self, target: Any, step: int) -> Path:
        path = self.path_for(step)
        exists = _agreed(path.exists())
        if exists and is_rank_zero():
            if path.is_dir():
                shutil.rmtree(path)
            else:
                path.unlink()
        _barrier()
        self.storage.write(path, target.state_dict(), after_write=self._prune)
        return path

    def _prune(self) -> None:
        c = self.config
        if c.keep_last_n < 0:
            return
        items = self._list()
        keep = {s for s, _ in items[-c.keep_last_n :]} if c.keep_last_n > 0 else set()
        for s, p in items:
            if s in keep or (c.keep_every and s % c.keep_every == 0):
                continue
            if p.is_dir():
                shutil.rmtree(p, ignore_errors=True)
            else:
                p.unlink(missing_ok=True)

    def flush(self) -> None:
        self.storage.flush()

    # ------------------------------------------------------------------ load
    def load(self, target: Any, max_steps: float = float("inf"), guard: bool = True) -> int | None:
        """Resume ``target`` from the newest complete checkpoint (or ``resume_step``).

        Returns the resumed step, or None. Falls back past unreadable checkpoints.
        """
        self.storage.flush()
        if not self.config.resume:
            if guard:
                self._guard_overwrite(0, max_steps)
            return None
        items = _agreed(self._list() if is_rank_zero() else None)
        if self.config.resume_step >= 0:
            items = [(s, p) for s, p in items if s == self.config.resume_step]
            if not items:
                raise FileNotFoundError(f"no complete checkpoint for step {self.config.resume_step} in {self.dir}")
        self._unreadable: set[int] = set()
        for step, path in reversed(items):
            try:
                state = self.storage.read(Path(path), target.state_dict())
            except Exception as exc:  # noqa: BLE001 -- fall back to an older checkpoint
                log.warning("checkpoint %s unreadable (%s); trying an older one", path, exc)
                self._unreadable.add(step)
                continue
            target.load_state_dict(state)
            if guard:
                self._guard_overwrite(step, max_steps)
            return step
        if guard:
            self._guard_overwrite(0, max_steps)
        return None

    def _guard_overwrite(self, start: int, max_steps: float) -> None:
        if self.config.allow_checkpoint_overwrite:
            return
        bad = getattr(self, "_unreadable", set())
        later = [s for s, _ in self._list() if s > start and s not in bad]
        if later and (max_steps == float("inf") or any(s <= max_steps for s in later)):
            raise RuntimeError(
                f"checkpoints after step {start} exist in {self.dir} ({later[:4]}...); this run would overwrite "
                "them. Set allow_checkpoint_overwrite=True to proceed."
            )
