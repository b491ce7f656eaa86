"""Download the nanochat corpus and fit its vocabulary (``priml/baselines/nanochat/scripts/prepare_data.py``).

    python -m priml_b200.baselines.nanochat.prepare_data [--directory DIR] [--vocab-size 8192]

1. Download: parquet text shards (the last is the validation shard), fetched
   once over plain HTTP and reused.
2. Fit: a byte-level BPE vocabulary on a prefix of the training text (each
   document capped at ``--tokenizer-doc-cap`` characters before it counts
   toward ``--tokenizer-train-chars``), with the 16 reserved tokens appended.
   The fit runs in this package's C++ trainer; a vocabulary whose recorded
   recipe matches the request is reused, anything else is refitted.

Rows are not packed here: packing is a stateful stream reproduced at read time
(:mod:`priml_b200.baselines.nanochat.data`).
"""

from __future__ import annotations

import argparse
import json
import logging
import urllib.request
from collections.abc import Iterator
from pathlib import Path
from typing import Any

from priml_b200.baselines.nanochat.data import BOS_TOKEN, SPLIT_PATTERN, fit_tokenizer

__all__ = ["prepare"]

log = logging.getLogger(__name__)

SOURCE_URL = "https://huggingface.co/datasets/karpathy/climbmix-400b-shuffle/resolve/main"


def _download(out: Path, count: int) -> list[Path]:
    out.mkdir(parents=True, exist_ok=True)
    paths = []
    for i in range(count):
        path = out / f"shard_{i:05d}.parquet"
        if not path.is_file():
            partial = path.with_suffix(".parquet.partial")
            log.info("downloading %s", path.name)
            urllib.request.urlretrieve(f"{SOURCE_URL}/shard_{i:05d}.parquet", partial)  # noqa: S310
            partial.replace(path)
        paths.append(path)
    return paths


def _documents(shards: list[Path], *, max_chars: int, doc_cap: int) -> Iterator[str]:
    from pyarrow import parquet

    seen = 0
    for path in shards:
        shard = parquet.ParquetFile(path)
        for group in range(shard.num_row_groups):
            for doc in shard.read_row_group(group).column("text").to_pylist():
                text = str(doc)[:doc_cap]
                seen += len(text)
                yield text
                if seen >= max_chars:
                    return


def prepare(directory: Path | str, *, num_train_shards: int = 7, vocab_size: int = 8192,
            tokenizer_train_chars: int = 2_000_000_000, tokenizer_doc_cap: int = 10_000, download: bool = True) -> None:  # fmt: skip
    """Download (unless ``download=False``: the shards must be present) and fit the vocabulary."""
    directory = Path(directory)
    names = [f"shard_{i:05d}.parquet" for i in range(num_train_shards + 1)]
    shards = _download(directory, num_train_shards + 1) if download else [directory / n for n in names]
    out = directory / "tokenizer"
    recipe: dict[str, Any] = {"vocab_size": vocab_size, "train_chars": tokenizer_train_chars,
                              "doc_cap": tokenizer_doc_cap, "shards": names[:num_train_shards],
                              "split_pattern": SPLIT_PATTERN, "bos_token": BOS_TOKEN}  # fmt: skip
    recipe_path = out / "tokenizer_recipe.json"
    if recipe_path.is_file() and (out / "bpe.json").is_file() and (out / "token_bytes.npy").is_file():
        recorded = json.loads(recipe_path.read_text())
        if all(recorded.get(k) == v for k, v in recipe.items()):
            log.info("nanochat vocabulary already fitted at %s", out)
            return
    log.info("fitting a %d-token vocabulary", vocab_size)
    docs = _documents(shards[:num_train_shards], max_chars=tokenizer_train_chars, doc_cap=tokenizer_doc_cap)
    tok = fit_tokenizer(docs, vocab_size=vocab_size, out=out, recipe=recipe)
    log.info("nanochat vocabulary fitted: %d tokens", tok.vocab_size)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--directory", default="/datasets/nanochat")
    ap.add_argument("--num-train-shards", type=int, default=7)
    ap.add_argument("--vocab-size", type=int, default=8192)
    ap.add_argument("--tokenizer-train-chars", type=int, default=2_000_000_000)
    ap.add_argument("--tokenizer-doc-cap", type=int, default=10_000)
    ap.add_argument("--no-download", action="store_true", help="fit on shards already in the directory")
    args = ap.parse_args()
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    prepare(args.directory, num_train_shards=args.num_train_shards, vocab_size=args.vocab_size,
            tokenizer_train_chars=args.tokenizer_train_chars, tokenizer_doc_cap=args.tokenizer_doc_cap,
            download=not args.no_download)  # fmt: skip
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
