"""One-line summaries of a run's metrics file (``priml/train/results.py:22-100``)."""

from __future__ import annotations

import argparse
import json
import sys
from collections.abc import Callable, Sequence
from pathlib import Path

__all__ = ["format_summary", "read_metrics", "summarize"]


def read_metrics(path: Path) -> dict[str, float]:
    """The metrics JSON object as ``{key: float}`` (raises if the file is missing)."""
    data = json.loads(Path(path).read_text())
    if not isinstance(data, dict):
        raise ValueError(f"{path} does not hold a JSON object")
    return {str(k): float(v) for k, v in data.items()}


def format_summary(metrics: dict[str, float], keys: Sequence[str] | None = None) -> str:
    """``key=value`` pairs (``eval/`` prefix dropped) in ``keys`` order or sorted."""
    chosen = list(keys) if keys is not None else sorted(metrics)
    parts = [f"{k.removeprefix('eval/')}={metrics[k]}" for k in chosen if k in metrics]
    return " ".join(parts) if parts else "no eval metrics found"


def summarize(argv: Sequence[str] | None = None, *, keys: Sequence[str] | None = None,
              note: Callable[[dict[str, float]], str] | None = None) -> int:  # fmt: skip
    """CLI: print the summary of ``--path`` (default ``metrics.json``); exit 1 if missing."""
    ap = argparse.ArgumentParser(description="Summarize a run's eval metrics.")
    ap.add_argument("--path", default="metrics.json")
    args = ap.parse_args(list(argv) if argv is not None else None)
    path = Path(args.path)
    if not path.exists():
        print(f"No metrics file at {path}.", file=sys.stderr)  # noqa: T201
        return 1
    metrics = read_metrics(path)
    line = format_summary(metrics, keys)
    if note is not None:
        line += note(metrics)
    print(line)  # noqa: T201
    return 0
