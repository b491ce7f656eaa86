"""Metric protocol: ``update(output, **batch)`` per eval batch, ``compute() -> dict``."""

from __future__ import annotations

import math

import pytest
import torch

from priml_b200.metrics import BinaryAccuracy, BitsPerByte, TopK


def test_topk_and_binary_accuracy() -> None:
    m = TopK(TopK.Config(k_values=[1, 2]))
    logits = torch.tensor([[0.1, 0.9, 0.0], [0.8, 0.1, 0.5], [0.2, 0.3, 0.9]])
    m.update(logits, label=torch.tensor([1, 2, 0]))
    assert m.compute() == {"top1": 1 / 3, "top2": 2 / 3}
    b = BinaryAccuracy()
    b.update(torch.tensor([[2.0], [-1.0], [0.5]]), label=torch.tensor([1, 0, 0]))
    assert b.compute() == {"accuracy": 2 / 3}


def test_bits_per_byte_skips_padding_rows_and_reserved_tokens() -> None:
    m = BitsPerByte()
    token_bytes = torch.tensor([1, 2, 3, 0])  # id 3 is a reserved token
    nats = torch.tensor([[1.0, 2.0], [4.0, 8.0], [100.0, 100.0]])
    label = torch.tensor([[0, 1], [2, 3], [1, 1]])
    m.update(nats, label=label, token_bytes=token_bytes, valid_count=2)  # row 2 is padding
    assert m.compute()["bpb"] == pytest.approx((1 + 2 + 4) / (math.log(2) * (1 + 2 + 3)))
    with pytest.raises(ValueError, match="no tokens"):
        BitsPerByte().compute()
