"""NanoChat data: parquet text shards, a byte-level BPE vocabulary, packed rows
(``priml/baselines/nanochat/data.py:88-786``).

A prepared directory holds::

    shard_00000.parquet ... shard_00007.parquet   text column "text"
    tokenizer/bpe.json                           merges, split pattern, reserved tokens
    tokenizer/token_bytes.npy                    [vocab_size] UTF-8 byte length per id
    tokenizer/tokenizer_recipe.json              what the vocabulary was fitted on

Rows are packed at read time exactly as the reference packs them: every
document starts with the BOS token, documents are placed largest-fits-first out
of a 1000-document buffer refilled 128 documents at a time, and when nothing
fits the shortest buffered document is cropped to fill the row. No padding.

Native pieces (``data/csrc/bpe.cpp``): the BPE merges (fit and encode, batches
on worker threads) and the packer run in C++; Python keeps the Unicode split
regex and the I/O. ``token_bytes.npy`` makes the score bits-per-byte: a
token's length is ``len(decode(token).encode())`` with replacement decoding,
the reference's rule, and reserved tokens count zero.
"""

from __future__ import annotations

import hashlib
import json
import logging
import queue
import threading
from collections.abc import Iterable, Iterator
from pathlib import Path
from typing import Any, Final

import numpy as np
import torch
from torch import Tensor

from priml_b200.config import Fig
from priml_b200.parallel.runtime import get_device

__all__ = [
    "BOS_TOKEN",
    "DOCUMENTS_PER_REFILL",
    "IGNORED_TARGET",
    "NanoChatData",
    "RESERVED_TOKENS",
    "SPLIT_PATTERN",
    "Tokenizer",
    "fit_tokenizer",
    "token_bytes_fingerprint",
]

log = logging.getLogger(__name__)

IGNORED_TARGET: Final = -1
"""Target the loss skips (no packed row carries it: packing leaves no padding)."""

DOCUMENTS_PER_REFILL: Final = 128
"""Documents encoded per buffer refill; part of the packing (best fit sees what the buffer holds)."""

SPLIT_PATTERN: Final = (
    r"""'(?i:[sdmt]|ll|ve|re)|[^\r\n\p{L}\p{N}]?+\p{L}+|\p{N}{1,2}"""
    r"""| ?[^\s\p{L}\p{N}]++[\r\n]*|\s*[\r\n]|\s+(?!\S)|\s+"""
)
"""Pre-split regex (numbers capped at two digits, a leading space kept with its word)."""

RESERVED_TOKENS: Final = tuple(f"<|reserved_{i}|>" for i in range(16))
BOS_TOKEN: Final = RESERVED_TOKENS[0]


def _native() -> Any:
    from priml_b200.data import _native  # type: ignore[attr-defined]

    return _native


def _splitter() -> Any:
    import regex

    return regex.compile(SPLIT_PATTERN)


def token_bytes_fingerprint(token_bytes: np.ndarray) -> str:
    """Hex SHA-256 of the byte-length table (canonical int64 bytes): the score's denominator."""
    return hashlib.sha256(np.ascontiguousarray(token_bytes, dtype=np.int64).tobytes()).hexdigest()


class Tokenizer:
    """Fitted byte-pair vocabulary plus reserved tokens, and the byte table that scores it."""

    def __init__(self, merges: list[tuple[int, int]], *, reserved: Iterable[str], bos_token: str,
                 token_bytes: np.ndarray | None = None) -> None:  # fmt: skip
        self.merges = [tuple(m) for m in merges]
        self.encoder = _native().BpeEncoder(self.merges)
        self.reserved = list(reserved)
        base = self.encoder.vocab_size()
        self.special = {name: base + i for i, name in enumerate(self.reserved)}
        self.bos_token_id = self.special[bos_token]
        self.bos_token = bos_token
        self._split = _splitter()
        self.token_bytes = token_bytes if token_bytes is not None else self._token_bytes()

    @property
    def vocab_size(self) -> int:
        return self.encoder.vocab_size() + len(self.reserved)

    def decode_bytes(self, ids: Iterable[int]) -> bytes:
        base = self.encoder.vocab_size()
        out = bytearray()
        for i in ids:
            out += self.reserved[i - base].encode() if i >= base else bytes(self.encoder.token_bytes(int(i)))
        return bytes(out)

    def decode(self, ids: Iterable[int]) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def _token_bytes(self) -> np.ndarray:
        base = self.encoder.vocab_size()
        lengths = [len(bytes(self.encoder.token_bytes(i)).decode("utf-8", errors="replace").encode()) for i in range(base)]
        return np.array(lengths + [0] * len(self.reserved), dtype=np.int32)

    def encode_ordinary(self, text: str) -> list[int]:
        return self.encode_batch([text], bos=False)[0]

    def encode_batch(self, texts: list[str], *, num_threads: int = 8, bos: bool = True) -> list[list[int]]:
        """Encode documents (each prefixed with BOS unless ``bos=False``)."""
        docs = [[c.encode("utf-8") for c in self._split.findall(t)] for t in texts]
        return self.encoder.encode_batch(docs, self.bos_token_id if bos else -1, num_threads)

    def save(self, directory: Path) -> None:
        directory.mkdir(parents=True, exist_ok=True)
        payload = {"merges": [list(m) for m in self.merges], "pattern": SPLIT_PATTERN, "reserved": self.reserved}
        staging = directory / "bpe.json.partial"
        staging.write_text(json.dumps(payload))
        staging.replace(directory / "bpe.json")
        np.save(directory / "token_bytes.npy", self.token_bytes)

    @classmethod
    def from_directory(cls, tokenizer_dir: Path | str) -> Tokenizer:
        """Load a prepared vocabulary, verified against the recipe recorded beside it."""
        tokenizer_dir = Path(tokenizer_dir)
        bpe, recipe_path = tokenizer_dir / "bpe.json", tokenizer_dir / "tokenizer_recipe.json"
        if not bpe.is_file() or not recipe_path.is_file():
            raise FileNotFoundError(
                f"no prepared nanochat vocabulary at {tokenizer_dir}; build it with "
                "`python -m priml_b200.baselines.nanochat.prepare_data`."
            )
        recipe = json.loads(recipe_path.read_text())
        for field_name in ("bos_token", "token_bytes_sha256"):
            if field_name not in recipe:
                raise ValueError(f"{recipe_path} declares no {field_name!r}; re-prepare the vocabulary.")
        raw = np.load(tokenizer_dir / "token_bytes.npy")
        if raw.ndim != 1 or not np.issubdtype(raw.dtype, np.integer):
            raise ValueError(f"{tokenizer_dir}/token_bytes.npy must be a 1-D integer table.")
        if recipe["token_bytes_sha256"] != token_bytes_fingerprint(raw):
            raise ValueError(f"{tokenizer_dir}: the byte table does not match its recorded fingerprint; re-prepare.")
        if int(raw.min(initial=0)) < 0:
            raise ValueError(f"{tokenizer_dir} holds a negative byte length.")
        payload = json.loads(bpe.read_text())
        tok = cls([tuple(m) for m in payload["merges"]], reserved=payload["reserved"], bos_token=recipe["bos_token"],
                  token_bytes=raw)  # fmt: skip
        if raw.shape[0] != tok.vocab_size:
            raise ValueError(f"{tokenizer_dir} fitted {tok.vocab_size} tokens but its byte table holds {raw.shape[0]}.")
        return tok


def fit_tokenizer(texts: Iterable[str], *, vocab_size: int, out: Path | str | None = None,
                  recipe: dict[str, Any] | None = None) -> Tokenizer:  # fmt: skip
    """Fit a byte-pair vocabulary of ``vocab_size`` ids (reserved tokens included) on ``texts``."""
    num_merges = vocab_size - 256 - len(RESERVED_TOKENS)
    if num_merges < 0:
        raise ValueError(f"vocab_size must be at least {256 + len(RESERVED_TOKENS)}; got {vocab_size}.")
    split = _splitter()
    trainer = _native().BpeTrainer()
    for text in texts:
        trainer.add_chunks([c.encode("utf-8") for c in split.findall(text)])
    merges = trainer.fit(num_merges)
    tok = Tokenizer(merges, reserved=RESERVED_TOKENS, bos_token=BOS_TOKEN)
    probe = "Hello world! Numbers: 123. Unicode: 你好"
    if tok.decode(tok.encode_ordinary(probe)) != probe:
        raise RuntimeError("the fitted vocabulary does not round-trip its probe text.")
    if out is not None:
        out = Path(out)
        tok.save(out)
        rec = dict(recipe or {})
        rec.update({"vocab_size": tok.vocab_size, "split_pattern": SPLIT_PATTERN, "bos_token": BOS_TOKEN,
                    "token_bytes_sha256": token_bytes_fingerprint(tok.token_bytes)})  # fmt: skip
        staging = out / "tokenizer_recipe.json.partial"
        staging.write_text(json.dumps(rec, sort_keys=True))
        staging.replace(out / "tokenizer_recipe.json")  # written last: it vouches for the files above
    return tok


def _document_batches(paths: list[Path]) -> Iterator[list[str]]:
    """Document batches of DOCUMENTS_PER_REFILL from parquet shards, wrapping at the end."""
    from pyarrow import parquet

    while True:
        for path in paths:
            shard = parquet.ParquetFile(path)
            for group in range(shard.num_row_groups):
                texts = shard.read_row_group(group).column("text").to_pylist()
                for start in range(0, len(texts), DOCUMENTS_PER_REFILL):
                    yield texts[start : start + DOCUMENTS_PER_REFILL]


def _shard_paths(directory: Path, indices: Iterable[int]) -> list[Path]:
    paths = [directory / f"shard_{i:05d}.parquet" for i in indices]
    missing = [p.name for p in paths if not p.is_file()]
    if missing:
        raise FileNotFoundError(f"{directory} is missing {missing}; prepare the corpus first.")
    return paths


class _PackedStream:
    """One split packed into ``[batch, max_seq_len + 1]`` rows, yielded as ``media`` / ``label`` views.

    The yielded tensors are views of reused buffers (consume before the next
    batch). With ``prefetch`` on CUDA a worker thread packs the next batch into
    one of two pinned staging slots while the current step runs; the host->
    device copy of a slot is recorded with an event the worker waits on before
    reusing the slot, so this thread never blocks on the device.
    """

    def __init__(self, *, paths: list[Path], tokenizer: Tokenizer, token_bytes: Tensor, batch_size: int,
                 max_seq_len: int, buffer_size: int, device: torch.device, max_batches: int | None,
                 prefetch: bool = False) -> None:  # fmt: skip
        self.paths, self.tokenizer, self.token_bytes = paths, tokenizer, token_bytes
        self.batch_size, self.max_seq_len, self.buffer_size = batch_size, max_seq_len, buffer_size
        self.device, self.max_batches, self.prefetch = device, max_batches, prefetch
        self.served = 0

    @property
    def _pins(self) -> bool:
        return self.device.type == "cuda" and torch.cuda.is_available()

    def __iter__(self) -> Iterator[dict[str, Any]]:
        return self._prefetched() if (self.prefetch and self._pins) else self._packed()

    def __len__(self) -> int:
        if self.max_batches is None:
            raise TypeError("the training stream is unbounded and has no length.")
        return self.max_batches

    def _rows(self) -> Iterator[np.ndarray]:
        """Packed ``[batch, max_seq_len + 1]`` int64 arrays, in the reference's order."""
        docs = _document_batches(self.paths)
        packer = _native().Packer(self.buffer_size, self.max_seq_len + 1)
        drawn = 0
        while self.max_batches is None or drawn < self.max_batches:
            rows = np.empty((self.batch_size, self.max_seq_len + 1), dtype=np.int64)
            while not packer.pack(rows):
                while packer.needs_refill():
                    packer.add(self.tokenizer.encode_batch(next(docs)))
            drawn += 1
            yield rows

    def _batch(self, media: Tensor, label: Tensor) -> dict[str, Any]:
        self.served += 1
        return {"media": media, "label": label, "token_bytes": self.token_bytes, "valid_count": self.batch_size}

    def _packed(self) -> Iterator[dict[str, Any]]:
        width = self.batch_size * self.max_seq_len
        pinned = self._pins
        staged = torch.empty(2 * width, dtype=torch.long, pin_memory=pinned)
        resident = torch.empty(2 * width, dtype=torch.long, device=self.device) if pinned else staged
        s_media = staged[:width].view(self.batch_size, self.max_seq_len)
        s_label = staged[width:].view(self.batch_size, self.max_seq_len)
        media = resident[:width].view(self.batch_size, self.max_seq_len)
        label = resident[width:].view(self.batch_size, self.max_seq_len)
        for rows in self._rows():
            r = torch.from_numpy(rows)
            s_media.copy_(r[:, :-1])
            s_label.copy_(r[:, 1:])
            if pinned:
                resident.copy_(staged, non_blocking=True)  # one transfer: inputs and targets back to back
            yield self._batch(media, label)

    def _prefetched(self) -> Iterator[dict[str, Any]]:
        width = self.batch_size * self.max_seq_len
        slots = [torch.empty(2 * width, dtype=torch.long, pin_memory=True) for _ in range(2)]
        resident = torch.empty(2 * width, dtype=torch.long, device=self.device)
        media = resident[:width].view(self.batch_size, self.max_seq_len)
        label = resident[width:].view(self.batch_size, self.max_seq_len)
        ready: queue.Queue[tuple[int, BaseException | None]] = queue.Queue(maxsize=1)
        done = threading.Event()
        free = [threading.Event() for _ in slots]
        for e in free:
            e.set()
        copied = [torch.cuda.Event() for _ in slots]

        def pack() -> None:
            slot = 0
            try:
                for rows in self._rows():
                    while not free[slot].wait(0.1):
                        if done.is_set():
                            return
                    copied[slot].synchronize()  # the slot's previous copy has landed
                    r = torch.from_numpy(rows)
                    buf = slots[slot]
                    buf[:width].view(self.batch_size, self.max_seq_len).copy_(r[:, :-1])
                    buf[width:].view(self.batch_size, self.max_seq_len).copy_(r[:, 1:])
                    free[slot].clear()
                    while not done.is_set():
                        try:
                            ready.put((slot, None), timeout=0.1)
                            break
                        except queue.Full:
                            continue
                    if done.is_set():
                        return
                    slot ^= 1
                ready.put((-1, None))
            except BaseException as exc:  # noqa: BLE001 -- handed to the consumer
                ready.put((-1, exc))

        worker = threading.Thread(target=pack, name="nanochat-pack", daemon=True)
        worker.start()
        try:
            while True:
                slot, err = ready.get()
                if err is not None:
                    raise err
                if slot < 0:
                    return
                resident.copy_(slots[slot], non_blocking=True)
                copied[slot].record()
                free[slot].set()
                yield self._batch(media, label)
        finally:
            done.set()
            worker.join(timeout=10)


class NanoChatData:
    """Prepared shards and vocabulary, served as packed ``media`` / ``label`` batches."""

    class Config(Fig["NanoChatData"]):
        working_dir: str = "/datasets/nanochat"
        tokenizer_dir: str = ""
        """Empty: ``<working_dir>/tokenizer``."""
        num_train_shards: int = 7
        val_shard: int = 7
        batch_size: int = 32
        eval_batch_size: int = 128
        eval_tokens: int = 40 * 524_288
        buffer_size: int = 1_000
        device: str | None = "auto"
        vocab_size: int = -1
        """Vocabulary the fitted tokenizer must report (-1: no check)."""
        max_seq_len: int = 2_048
        prefetch: bool = True

    def __init__(self, config: Config | None = None) -> None:
        config = config or NanoChatData.Config()
        if min(config.batch_size, config.eval_batch_size, config.buffer_size) <= 0:
            raise ValueError("batch sizes and buffer_size must be positive.")
        if config.max_seq_len < 2:
            raise ValueError(f"max_seq_len must be at least two; got {config.max_seq_len}.")
        per_eval = config.eval_batch_size * config.max_seq_len
        if config.eval_tokens <= 0 or config.eval_tokens % per_eval:
            raise ValueError(f"eval_tokens={config.eval_tokens} must be a positive multiple of {per_eval}.")
        self.config = config
        self.device = get_device(config.device)
        self.dataset_dir = Path(config.working_dir)
        self.train_paths = _shard_paths(self.dataset_dir, range(config.num_train_shards))
        self.val_paths = _shard_paths(self.dataset_dir, [config.val_shard])
        self.tokenizer = Tokenizer.from_directory(Path(config.tokenizer_dir or self.dataset_dir / "tokenizer"))
        if 0 < config.vocab_size != self.tokenizer.vocab_size:
            raise ValueError(
                f"the fitted vocabulary holds {self.tokenizer.vocab_size} tokens but the model declares "
                f"vocab_size {config.vocab_size}."
            )
        self.token_bytes = torch.from_numpy(self.tokenizer.token_bytes.astype(np.int32)).to(self.device)
        self._live: _PackedStream | None = None

    def _stream(self, paths: list[Path], batch: int, max_batches: int | None, prefetch: bool) -> _PackedStream:
        c = self.config
        return _PackedStream(paths=paths, tokenizer=self.tokenizer, token_bytes=self.token_bytes, batch_size=batch,
                             max_seq_len=c.max_seq_len, buffer_size=c.buffer_size, device=self.device,
                             max_batches=max_batches, prefetch=prefetch)  # fmt: skip

    def train_dataloader(self) -> _PackedStream:
        """The training stream: the corpus, packed, without end."""
        self._live = self._stream(self.train_paths, self.config.batch_size, None, self.config.prefetch)
        return self._live

    def eval_dataloader(self) -> _PackedStream:
        """The pinned validation shard from its start, capped at ``eval_tokens``."""
        c = self.config
        return self._stream(self.val_paths, c.eval_batch_size, c.eval_tokens // (c.eval_batch_size * c.max_seq_len), False)

    def state_dict(self) -> dict[str, Any]:
        return {"batches": self._live.served if self._live is not None else 0}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        served = int(state_dict.get("batches", 0))
        if served:
            raise ValueError(
                f"this checkpoint had served {served} batches; the packed stream cannot be positioned without "
                "re-tokenizing the corpus up to that point. Start a fresh run."
            )
