"""Static-cache decoding and device-side sampling on CPU, against the reference-style loop.

* :class:`Decoder` greedy output equals :func:`priml_b200.models.generate.generate`
  (the reference's ``generate`` port) and the full forward's argmax;
* refilling one row and appending a chunk to a partly filled row give the full
  forward's logits;
* the decode-attention oracle hides keys past each row's length and outside the window;
* the Gumbel-max sampler draws ``softmax(z / T)`` after top-k / top-p filtering.
"""

from __future__ import annotations

import pytest
import torch

from priml_b200.inference import Decoder, SamplingParams, sample
from priml_b200.models.generate import generate
from priml_b200.models.presets import tiny_lm


@pytest.fixture(scope="module")
def model() -> torch.nn.Module:
    torch.manual_seed(0)
    return tiny_lm().make().eval()


def test_greedy_decoder_matches_generate_and_full_forward(model: torch.nn.Module) -> None:
    prompt = torch.randint(0, 512, (3, 7), generator=torch.Generator().manual_seed(1))
    ref = generate(model, prompt, max_new_tokens=10, temperature=0, max_seq_len=64)
    out = Decoder(model, batch=3, max_seq=64).generate(prompt, max_new_tokens=10, temperature=0)
    assert out.tolist() == ref.tolist()
    with torch.no_grad():
        full = model(out[:, :-1])
    assert torch.equal(full[:, 6:].argmax(-1), out[:, 7:])


def test_row_refill_and_chunk_append(model: torch.nn.Module) -> None:
    prompts = torch.randint(0, 512, (2, 9), generator=torch.Generator().manual_seed(2))
    dec = Decoder(model, batch=2, max_seq=32)
    dec.prefill(prompts)
    dec.step(torch.tensor([5, 6]))
    dec.reset(slice(1, 2))  # row 0 keeps its cache
    first = dec.prefill(prompts[1:, :4], rows=slice(1, 2))
    rest = dec.prefill(prompts[1:, 4:], rows=slice(1, 2))
    with torch.no_grad():
        torch.testing.assert_close(first, model(prompts[1:, :4])[:, -1], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(rest, model(prompts[1:])[:, -1], rtol=1e-5, atol=1e-5)
        _, logits = dec.step(torch.tensor([7, 8]))
        row0 = model(torch.cat([prompts[:1], torch.tensor([[5, 7]])], dim=1))[:, -1]
        torch.testing.assert_close(logits[:1], row0, rtol=1e-5, atol=1e-5)
    assert dec.host_lengths == [11, 10]


def test_cache_overflow_is_refused(model: torch.nn.Module) -> None:
    dec = Decoder(model, batch=1, max_seq=8)
    dec.prefill(torch.zeros(1, 8, dtype=torch.long))
    with pytest.raises(ValueError, match="overflow"):
        dec.step(torch.zeros(1, dtype=torch.long))


def test_decode_attention_oracle_masks_length_and_window() -> None:
    from priml_b200 import ops

    torch.manual_seed(3)
    q = torch.randn(3, 4, 16)
    k, v = torch.randn(3, 2, 10, 16), torch.randn(3, 2, 10, 16)
    lengths = torch.tensor([10, 4, 0])
    out = ops.decode_attention(q, k, v, lengths, window=2)
    for b, n in enumerate(lengths.tolist()):
        for h in range(4):
            if n == 0:
                assert out[b, h].abs().max() == 0
                continue
            lo = max(0, n - 3)
            s = (k[b, h // 2, lo:n] @ q[b, h]) / 4.0
            torch.testing.assert_close(out[b, h], s.softmax(-1) @ v[b, h // 2, lo:n], rtol=1e-5, atol=1e-5)


def test_sampler_greedy_topk_topp_and_distribution() -> None:
    torch.manual_seed(4)
    logits = torch.randn(4, 50)
    params = [SamplingParams(0.0), SamplingParams(1.0, top_k=1), SamplingParams(1.0, top_p=1e-6),
              SamplingParams(0.7, top_k=5, top_p=0.9)]  # fmt: skip
    t, k, p = SamplingParams.stack(params)
    tok = sample(logits, t, k, p)
    greedy = logits.argmax(-1)
    assert tok[:3].tolist() == greedy[:3].tolist()
    top5 = logits[3].topk(5).indices.tolist()
    assert int(tok[3]) in top5

    # Gumbel-max draws follow softmax(z / T): frequencies over many rows
    z = torch.tensor([2.0, 1.0, 0.0, -1.0])
    n = 40000
    rows = z.expand(n, 4)
    g = torch.Generator().manual_seed(5)
    temp = torch.full((n,), 0.8)
    draws = sample(rows, temp, torch.zeros(n, dtype=torch.long), torch.ones(n), filtered=False, generator=g)
    freq = torch.bincount(draws, minlength=4).float() / n
    torch.testing.assert_close(freq, (z / 0.8).softmax(-1), rtol=0, atol=0.01)

    # top-p keeps the smallest prefix whose exclusive mass is within p: here the first two tokens
    draws = sample(rows, torch.ones(n), torch.zeros(n, dtype=torch.long), torch.full((n,), 0.7), generator=g)
    freq = torch.bincount(draws, minlength=4).float() / n
    kept = z[:2].softmax(-1)
    torch.testing.assert_close(freq, torch.cat([kept, torch.zeros(2)]), rtol=0, atol=0.01)
