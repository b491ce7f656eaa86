"""Build the Sudoku-Extreme splits (``priml/baselines/sudoku/scripts/prepare_data.py:1-353``).

``python -m priml_b200.baselines.sudoku.prepare_data [--directory D] [--csv-directory C]``

The source is the Sudoku-Extreme CSV pair at a pinned revision, verified by
SHA-256 before parsing (the same bytes the reference trains on). Training keeps
``num_puzzles`` puzzles drawn without replacement and writes each followed by
``copies_per_puzzle`` validity-preserving transforms: a digit relabeling, an
optional transpose, a shuffle of the three bands and of the rows within each
band, and the same for stacks and columns. The test split is written as is.

Grids are tokenized as ``digit + 1`` (blank = 1). With ``--csv-directory`` the
CSVs are read locally instead of downloaded (this machine has no network).
"""

from __future__ import annotations

import argparse
import csv
import hashlib
import json
import logging
import shutil
import tempfile
import urllib.request
from collections.abc import Sequence
from pathlib import Path
from typing import Final

import numpy as np

log = logging.getLogger(__name__)

__all__ = ["SOURCE_REVISION", "SOURCE_SHA256", "prepare", "transform", "write_split"]

SOURCE_URL: Final = "https://huggingface.co/datasets/sapientinc/sudoku-extreme/resolve"
SOURCE_REVISION: Final = "58942f96baeb572ca3127e2a9e9c70f330783d6b"
SOURCE_SHA256: Final = {
    "train.csv": "64b46674db0148e0d73a16346dadeb2b1c00824d3fca3f85b2ae7037f6b4b38e",
    "test.csv": "a2fd52aea23d331d5b4ee723c856236e838a9fb9a70e66f4e0e0cf26c338c6a8",
}
N: Final = 9
BOX: Final = 3
VOCAB_SIZE: Final = 11


def transform(puzzle: np.ndarray, solution: np.ndarray, rng: np.random.Generator) -> tuple[np.ndarray, np.ndarray]:
    """One random validity-preserving transform applied identically to a ``[9, 9]`` puzzle and its solution."""
    relabel = np.concatenate([[0], rng.permutation(np.arange(1, N + 1))])
    flip = rng.random() < 0.5
    row_order = np.concatenate([band * BOX + rng.permutation(BOX) for band in rng.permutation(BOX)])
    col_order = np.concatenate([stack * BOX + rng.permutation(BOX) for stack in rng.permutation(BOX)])

    def apply(g: np.ndarray) -> np.ndarray:
        g = g.T if flip else g
        return relabel[g[np.ix_(row_order, col_order)]]

    return apply(puzzle), apply(solution)


def write_split(destination: Path | str, puzzles: Sequence[np.ndarray], solutions: Sequence[np.ndarray], *,
                copies_per_puzzle: int, rng: np.random.Generator) -> None:  # fmt: skip
    """Write one split: every puzzle then its transformed copies, contiguous, with row bounds."""
    out = Path(destination)
    inputs, labels, bounds = [], [], [0]
    for p, s in zip(puzzles, solutions, strict=True):
        inputs.append(p.reshape(-1))
        labels.append(s.reshape(-1))
        for _ in range(copies_per_puzzle):
            tp, ts = transform(p, s, rng)
            inputs.append(tp.reshape(-1))
            labels.append(ts.reshape(-1))
        bounds.append(len(inputs))
    x, y = np.stack(inputs), np.stack(labels)
    if x.min() < 0 or x.max() > N or y.min() < 0 or y.max() > N:
        raise ValueError("grid cells must hold 0 (blank) .. 9")
    out.mkdir(parents=True, exist_ok=True)
    np.save(out / "all__inputs.npy", (x + 1).astype(np.int32))
    np.save(out / "all__labels.npy", (y + 1).astype(np.int32))
    np.save(out / "all__group_indices.npy", np.asarray(bounds, dtype=np.int32))
    (out / "dataset.json").write_text(json.dumps({"vocab_size": VOCAB_SIZE, "seq_len": N * N}))


def _grid(text: str) -> np.ndarray:
    return (np.frombuffer(text.encode(), dtype=np.uint8).reshape(N, N) - ord("0")).astype(np.int64)


def _read_csv(path: Path) -> tuple[list[np.ndarray], list[np.ndarray]]:
    puzzles, solutions = [], []
    with path.open(newline="") as f:
        rows = csv.reader(f)
        next(rows)  # header: source, question, answer, rating
        for _source, question, answer, _rating in rows:
            puzzles.append(_grid(question.replace(".", "0")))
            solutions.append(_grid(answer))
    return puzzles, solutions


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _download(name: str, into: Path) -> Path:
    into.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=into, prefix=f".{name}.", suffix=".part")
    path = Path(tmp)
    with urllib.request.urlopen(f"{SOURCE_URL}/{SOURCE_REVISION}/{name}") as r, open(fd, "wb") as f:
        shutil.copyfileobj(r, f)
    return path


def prepare(directory: Path | str, *, num_puzzles: int = 1000, copies_per_puzzle: int = 1000, seed: int = 42,
            csv_directory: Path | str | None = None) -> Path:  # fmt: skip
    out = Path(directory)
    rng = np.random.default_rng(seed)
    for split in ("train", "test"):
        if (out / split / "dataset.json").is_file():
            log.info("sudoku %s already prepared", split)
            continue
        name = f"{split}.csv"
        fetched = None
        if csv_directory is not None:
            src = Path(csv_directory) / name
        else:
            src = fetched = _download(name, out)
        digest = _sha256(src)
        if digest != SOURCE_SHA256[name]:
            raise RuntimeError(f"{src} has SHA-256 {digest}; revision {SOURCE_REVISION} needs {SOURCE_SHA256[name]}.")
        puzzles, solutions = _read_csv(src)
        if split == "train" and num_puzzles < len(puzzles):
            keep = rng.choice(len(puzzles), size=num_puzzles, replace=False)
            puzzles = [puzzles[int(i)] for i in keep]
            solutions = [solutions[int(i)] for i in keep]
        write_split(out / split, puzzles, solutions, copies_per_puzzle=copies_per_puzzle if split == "train" else 0,
                    rng=rng)  # fmt: skip
        if fetched is not None:
            fetched.unlink(missing_ok=True)
        log.info("sudoku %s: %d puzzles", split, len(puzzles))
    return out


def main(argv: Sequence[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Prepare the Sudoku-Extreme splits.")
    ap.add_argument("--directory", default="datasets/sudoku-extreme")
    ap.add_argument("--csv-directory", default=None)
    ap.add_argument("--num-puzzles", type=int, default=1000)
    ap.add_argument("--copies-per-puzzle", type=int, default=1000)
    ap.add_argument("--seed", type=int, default=42)
    a = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    prepare(a.directory, num_puzzles=a.num_puzzles, copies_per_puzzle=a.copies_per_puzzle, seed=a.seed,
            csv_directory=a.csv_directory)  # fmt: skip
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
