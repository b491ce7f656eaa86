"""NanoChat baseline: native BPE + packer, data stream, model and budgeted train step (CPU)."""

from __future__ import annotations

import random
from pathlib import Path

import numpy as np
import pytest
import torch


def _py_pack_row(row: list[int], buffer: list[list[int]], position: int) -> int:
    """The packing rule, restated in Python: largest document that fits, else crop the shortest."""
    remaining = len(row) - position
    best, best_len = -1, 0
    for i, d in enumerate(buffer):
        if best_len < len(d) <= remaining:
            best, best_len = i, len(d)
    if best >= 0:
        d = buffer.pop(best)
        row[position : position + len(d)] = d
        return position + len(d)
    shortest = min(range(len(buffer)), key=lambda i: len(buffer[i]))
    d = buffer.pop(shortest)
    row[position : position + remaining] = d[:remaining]
    return position + remaining


def test_native_packer_matches_the_packing_rule() -> None:
    from priml_b200.data import _native

    rng = random.Random(0)
    docs = [[rng.randrange(1000) for _ in range(rng.randrange(1, 90))] for _ in range(3000)]
    buffer_size, row_len, batch = 20, 64, 4
    # Python restatement
    it, buf, want = iter(docs), [], []
    for _ in range(5):
        rows = []
        for _ in range(batch):
            row, pos = [0] * row_len, 0
            while pos < row_len:
                while len(buf) < buffer_size:
                    buf.extend([next(it) for _ in range(7)])
                pos = _py_pack_row(row, buf, pos)
            rows.append(row)
        want.append(rows)
    # native
    it = iter(docs)
    packer = _native.Packer(buffer_size, row_len)
    got = []
    for _ in range(5):
        out = np.empty((batch, row_len), dtype=np.int64)
        while not packer.pack(out):
            while packer.needs_refill():
                packer.add([next(it) for _ in range(7)])
        got.append(out.tolist())
    assert got == want


def test_bpe_fit_encode_roundtrip_and_byte_table(tmp_path: Path) -> None:
    from priml_b200.baselines.nanochat.data import RESERVED_TOKENS, Tokenizer, fit_tokenizer

    texts = ["the quick brown fox jumps over the lazy dog " * 20, "hello world 12345 你好 " * 30, "don't stop, we're fine"] * 5
    tok = fit_tokenizer(texts, vocab_size=256 + 16 + 40, out=tmp_path, recipe={"shards": []})
    assert tok.vocab_size == 256 + 40 + len(RESERVED_TOKENS)
    for t in texts[:3] + ["unseen text ✓ 987"]:
        ids = tok.encode_ordinary(t)
        assert tok.decode(ids) == t
    # merges shorten the encoding of the fitted text
    assert len(tok.encode_ordinary(texts[0])) < len(texts[0].encode()) / 2
    # byte table: reserved tokens are zero, merged tokens their UTF-8 length
    assert tok.token_bytes[-16:].sum() == 0 and tok.token_bytes[ord("a")] == 1
    loaded = Tokenizer.from_directory(tmp_path)
    assert loaded.encode_batch(texts[:2]) == tok.encode_batch(texts[:2])
    assert loaded.encode_batch(["x"])[0][0] == loaded.bos_token_id
    np.save(tmp_path / "token_bytes.npy", loaded.token_bytes + 1)  # tampered denominator
    with pytest.raises(ValueError, match="fingerprint"):
        Tokenizer.from_directory(tmp_path)


def _corpus(tmp_path: Path, shards: int = 3) -> None:
    import pyarrow as pa
    import pyarrow.parquet as pq

    rng = random.Random(1)
    words = ["alpha", "beta", "gamma", "delta", "token", "stream", "packing", "row", "the", "of"]
    for s in range(shards):
        docs = [" ".join(rng.choice(words) for _ in range(rng.randrange(3, 60))) for _ in range(300)]
        pq.write_table(pa.table({"text": docs}), tmp_path / f"shard_{s:05d}.parquet", row_group_size=100)
    from priml_b200.baselines.nanochat.data import fit_tokenizer

    fit_tokenizer(docs, vocab_size=256 + 16 + 64, out=tmp_path / "tokenizer", recipe={"shards": ["x"]})


def test_stream_batches_rows_with_bos_and_shifted_labels(tmp_path: Path) -> None:
    from priml_b200.baselines.nanochat.data import NanoChatData

    _corpus(tmp_path)
    data = NanoChatData(NanoChatData.Config(working_dir=str(tmp_path), num_train_shards=2, val_shard=2, batch_size=3,
                                            eval_batch_size=2, eval_tokens=2 * 32 * 3, max_seq_len=32,
                                            buffer_size=50, device="cpu"))  # fmt: skip
    it = iter(data.train_dataloader())
    b = next(it)
    assert b["media"].shape == (3, 32) and torch.equal(b["media"][:, 1:], b["label"][:, :-1])
    assert int(b["media"][0, 0]) == data.tokenizer.bos_token_id  # every row starts a document
    assert len(list(data.eval_dataloader())) == 3
    assert data.state_dict()["batches"] == 1
    with pytest.raises(ValueError, match="cannot be positioned"):
        data.load_state_dict({"batches": 5})


def test_nanochat_step_trains_on_the_stream(tmp_path: Path) -> None:
    from priml_b200.baselines.nanochat import NanoChatLM, NanoChatTrainStep, nanochat_optimizer
    from priml_b200.baselines.nanochat.data import NanoChatData
    from priml_b200.models.swiglu import SwiGLUReluSquared
    from priml_b200.models.transformer import TransformerBlock
    from priml_b200.models.value_gated_attention import ValueGatedAttention

    _corpus(tmp_path)
    data = NanoChatData(NanoChatData.Config(working_dir=str(tmp_path), num_train_shards=2, val_shard=2, batch_size=4,
                                            eval_batch_size=4, eval_tokens=4 * 64, max_seq_len=64, device="cpu"))  # fmt: skip
    torch.manual_seed(0)
    model = NanoChatLM.Config(vocab_size=data.tokenizer.vocab_size, max_seq_len=64, channels_in=64, num_layers=4,
                              value_embedding_stride=2,
                              block=TransformerBlock.Config(attn=ValueGatedAttention.Config(channels_head=32),
                                                            ffn=SwiGLUReluSquared.Config()))  # fmt: skip
    step = NanoChatTrainStep.Config(model=model, optimizer=nanochat_optimizer(compile=False), dtype_autocast=None,
                                    tokens_per_optimizer_step=2 * 4 * 64, rows_per_pass=4, budget_warmup_steps=0,
                                    train_budget_sec=120.0).make()  # fmt: skip
    assert sorted(step.model.value_embeds) == ["1", "3"]
    assert [b.attn.config.window for b in step.model.blocks][-1] == 64
    losses = []
    it = iter(data.train_dataloader())
    for _ in range(16):
        out = step.train_step(**next(it))
        if out["stepped"]:
            losses.append(float(out["loss"]))
    assert len(losses) == 8 and all(np.isfinite(losses))
    assert losses[-1] < losses[0]
    ev = step.eval_loss(**next(iter(data.eval_dataloader())))
    assert ev["model"].shape == (4, 64)
    # fused loss == the logits path
    b = next(it)
    with torch.no_grad():
        fused = step.model.token_loss(b["media"], b["label"])
        logits = step.model(b["media"])
        ref = torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), b["label"].reshape(-1),
                                                reduction="none").view(b["label"].shape)  # fmt: skip
    torch.testing.assert_close(fused, ref, rtol=1e-4, atol=1e-4)
    sd = step.state_dict()
    assert "elapsed_sec" in sd and sd["local_step"] == 8


def test_smoke_experiment_runs_the_loop_end_to_end(tmp_path: Path) -> None:
    from priml_b200.baselines.nanochat.data import Tokenizer
    from priml_b200.baselines.nanochat.experiments import exp000, exp003, exp_smoke

    _corpus(tmp_path)
    vocab = Tokenizer.from_directory(tmp_path / "tokenizer").vocab_size
    cfg = exp_smoke()
    cfg.working_dir = str(tmp_path / "run")
    cfg.dataset.working_dir = str(tmp_path)
    cfg.dataset.num_train_shards, cfg.dataset.val_shard = 2, 2
    cfg.dataset.device = "cpu"
    cfg.dataset.prefetch = False
    cfg.step.model.vocab_size = vocab
    cfg.step.dtype_autocast = None
    cfg.step.optimizer.optimizers[-1].compile = False
    loop = cfg.make()
    result = loop.train()
    assert loop.global_step == 4
    assert 0.0 < result["eval/val_bpb"] < 20.0  # bits per byte of an untrained model
    # the recipe rungs build (without data) and differ where they say they do
    assert exp003().step.model.value_embedding_stride == 0
    assert exp000().step.model.value_embedding_stride == 2


def test_prepare_fits_once_and_reuses_a_matching_vocabulary(tmp_path: Path) -> None:
    from priml_b200.baselines.nanochat.data import NanoChatData
    from priml_b200.baselines.nanochat.prepare_data import prepare

    _corpus(tmp_path, shards=3)
    prepare(tmp_path, num_train_shards=2, vocab_size=256 + 16 + 32, tokenizer_train_chars=50_000, download=False)
    stamp = (tmp_path / "tokenizer" / "bpe.json").stat().st_mtime_ns
    prepare(tmp_path, num_train_shards=2, vocab_size=256 + 16 + 32, tokenizer_train_chars=50_000, download=False)
    assert (tmp_path / "tokenizer" / "bpe.json").stat().st_mtime_ns == stamp  # reused, not refitted
    data = NanoChatData(NanoChatData.Config(working_dir=str(tmp_path), num_train_shards=2, val_shard=2, batch_size=2,
                                            eval_batch_size=2, eval_tokens=2 * 16, max_seq_len=16,
                                            vocab_size=256 + 16 + 32, device="cpu"))  # fmt: skip
    assert data.tokenizer.vocab_size == 256 + 16 + 32
