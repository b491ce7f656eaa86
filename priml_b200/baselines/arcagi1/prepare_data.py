"""Build the ARC-AGI-1 splits from task JSON files.

``python -m priml_b200.baselines.arcagi1.prepare_data --tasks-directory ARC/data --directory D``

``--tasks-directory`` holds ``training/`` and ``evaluation/`` folders of ARC
task files (``{"train": [{"input", "output"}...], "test": [...]}``). Every task
is expanded into ``views`` puzzles: the identity plus random distinct views,
each a square symmetry (one of 8) composed with a permutation of colors 1..9
(black stays black). Each view is one puzzle with its own identifier, i.e. one
row of the sparse per-puzzle table.

* ``train`` split: every pair of every training task, and the DEMONSTRATION
  pairs of every evaluation task (so each evaluation view's identifier is
  trained);
* ``test`` split: the evaluation tasks' test pairs under the same views and
  identifiers.

Grids are placed at the top-left of a 30 x 30 canvas: color ``c`` is token
``c + 2``, the row below and the column right of the grid carry the end
marker 1, everything else is pad 0 (the label's ignore id). Rows, puzzles and
tasks are written in the layout :class:`ArcData` reads.
"""

from __future__ import annotations

import argparse
import json
import logging
from collections.abc import Sequence
from pathlib import Path
from typing import Any

import numpy as np

__all__ = ["SIDE", "encode_grid", "prepare", "view_transform"]

log = logging.getLogger(__name__)

SIDE = 30
VOCAB_SIZE = 12


def encode_grid(grid: np.ndarray) -> np.ndarray:
    """``[h, w]`` colors -> flat ``[900]`` tokens with end markers and pad."""
    h, w = grid.shape
    if h > SIDE or w > SIDE:
        raise ValueError(f"grid {h}x{w} exceeds {SIDE}x{SIDE}")
    canvas = np.zeros((SIDE, SIDE), dtype=np.int32)
    canvas[:h, :w] = grid + 2
    if h < SIDE:
        canvas[h, : min(w + 1, SIDE)] = 1
    if w < SIDE:
        canvas[: min(h + 1, SIDE), w] = 1
    return canvas.reshape(-1)


def view_transform(grid: np.ndarray, symmetry: int, colors: np.ndarray) -> np.ndarray:
    """Square symmetry ``symmetry`` (rotation ``symmetry // 2``, mirrored when odd) then recoloring."""
    g = np.rot90(grid, symmetry // 2)
    if symmetry % 2:
        g = g[:, ::-1]
    return colors[g]


def _views(rng: np.random.Generator, count: int) -> list[tuple[int, np.ndarray]]:
    out = [(0, np.arange(10))]
    seen = {(0, tuple(range(10)))}
    while len(out) < count:
        colors = np.concatenate([[0], 1 + rng.permutation(9)])
        key = (int(rng.integers(8)), tuple(int(c) for c in colors))
        if key not in seen:
            seen.add(key)
            out.append((key[0], colors))
    return out


def _load(directory: Path) -> list[dict[str, Any]]:
    return [json.loads(p.read_text()) for p in sorted(directory.glob("*.json"))]


def _write(destination: Path, tasks: list[list[list[tuple[np.ndarray, np.ndarray]]]], ids: list[list[int]],
           num_ids: int) -> None:  # fmt: skip
    """``tasks[t][v]`` is the list of (input, output) pairs of view ``v`` of task ``t``."""
    inputs, labels, puzzle_bounds, group_bounds, identifiers = [], [], [0], [0], []
    for views, view_ids in zip(tasks, ids, strict=True):
        for pairs, pid in zip(views, view_ids, strict=True):
            for x, y in pairs:
                inputs.append(encode_grid(x))
                labels.append(encode_grid(y))
            puzzle_bounds.append(len(inputs))
            identifiers.append(pid)
        group_bounds.append(len(identifiers))
    destination.mkdir(parents=True, exist_ok=True)
    np.save(destination / "all__inputs.npy", np.stack(inputs).astype(np.int32))
    np.save(destination / "all__labels.npy", np.stack(labels).astype(np.int32))
    np.save(destination / "all__puzzle_indices.npy", np.asarray(puzzle_bounds, dtype=np.int32))
    np.save(destination / "all__group_indices.npy", np.asarray(group_bounds, dtype=np.int32))
    np.save(destination / "all__puzzle_identifiers.npy", np.asarray(identifiers, dtype=np.int32))
    (destination / "dataset.json").write_text(json.dumps({"vocab_size": VOCAB_SIZE, "seq_len": SIDE * SIDE,
                                                          "ignore_label_id": 0,
                                                          "num_puzzle_identifiers": num_ids}))  # fmt: skip


def prepare(directory: Path | str, *, training: Sequence[dict[str, Any]], evaluation: Sequence[dict[str, Any]],
            views: int = 8, seed: int = 0) -> Path:  # fmt: skip
    """Write ``train/`` and ``test/`` under ``directory`` from already-parsed task dicts."""
    rng = np.random.default_rng(seed)
    out = Path(directory)
    train_tasks, train_ids, test_tasks, test_ids = [], [], [], []
    next_id = 0

    def pairs(task: dict[str, Any], key: str, sym: int, colors: np.ndarray) -> list[tuple[np.ndarray, np.ndarray]]:
        return [(view_transform(np.asarray(p["input"]), sym, colors), view_transform(np.asarray(p["output"]), sym, colors))
                for p in task.get(key, []) if "output" in p]  # fmt: skip

    for task in training:
        vs = _views(rng, views)
        train_tasks.append([pairs(task, "train", s, c) + pairs(task, "test", s, c) for s, c in vs])
        train_ids.append(list(range(next_id, next_id + len(vs))))
        next_id += len(vs)
    for task in evaluation:
        vs = _views(rng, views)
        ids = list(range(next_id, next_id + len(vs)))
        next_id += len(vs)
        train_tasks.append([pairs(task, "train", s, c) for s, c in vs])
        train_ids.append(ids)
        test_tasks.append([pairs(task, "test", s, c) for s, c in vs])
        test_ids.append(ids)
    _write(out / "train", train_tasks, train_ids, next_id)
    _write(out / "test", test_tasks, test_ids, next_id)
    log.info("ARC: %d training + %d evaluation tasks, %d views each, %d identifiers",
             len(training), len(evaluation), views, next_id)  # fmt: skip
    return out


def main(argv: Sequence[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Prepare the ARC-AGI-1 splits from task JSON files.")
    ap.add_argument("--tasks-directory", required=True, help="folder with training/ and evaluation/ task files")
    ap.add_argument("--directory", default="datasets/arcagi1")
    ap.add_argument("--views", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    src = Path(a.tasks_directory)
    prepare(a.directory, training=_load(src / "training"), evaluation=_load(src / "evaluation"), views=a.views,
            seed=a.seed)  # fmt: skip
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
