"""Machine-readable progress file (``priml/train/progress.py:20-70``)."""

from __future__ import annotations

import json
import os
from datetime import UTC, datetime
from pathlib import Path

__all__ = ["write_progress"]


def write_progress(step: int, total: int, *, working_dir: Path | str, metrics: dict[str, float] | None = None) -> Path:
    """Atomically replace ``<working_dir>/progress.json`` with ``{step, total, metrics, updated_at}``.

    Every writer (e.g. each torchrun rank) uses its own temporary name, so a
    reader never sees a torn file and concurrent writers never rename each
    other's half-written files.
    """
    if not working_dir:
        raise ValueError("working_dir must not be empty")
    path = Path(working_dir) / "progress.json"
    path.parent.mkdir(parents=True, exist_ok=True)
    payload = {
        "step": int(step),
        "total": int(total),
        "metrics": {k: float(v) for k, v in (metrics or {}).items()},
        "updated_at": datetime.now(tz=UTC).strftime("%Y-%m-%dT%H:%M:%SZ"),
    }
    tmp = path.with_name(f"progress.json.{os.getpid()}.tmp")
    tmp.write_text(json.dumps(payload))
    os.replace(tmp, path)
    return path
