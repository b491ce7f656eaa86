"""Autoregressive sampling with per-block KV caches (``priml/model/generate.py:40-188``).

Prefill runs the whole prompt once; each decode step feeds one token through
every block with its cache. Sampling follows the HF conventions (temperature,
top-k, then top-p on the exclusive cumulative mass).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

__all__ = ["generate", "sample_logits"]


def _run_blocks(model: Any, x: Tensor, caches: list[Any]) -> Tensor:
    for i, block in enumerate(model.blocks):
        res = block(x, cache=caches[i])
        if isinstance(res, tuple):
            x, caches[i] = res
        else:
            x = res
    return x


@torch.inference_mode()
def generate(
    model: Any,
    prompt_ids: Tensor,
    *,
    max_new_tokens: int = 128,
    temperature: float = 1.0,
    top_k: int = 0,
    top_p: float = 1.0,
    eos_token_id: int | None = None,
    max_seq_len: int = 1024,
) -> Tensor:
    """``(B, S)`` prompt -> ``(B, S + generated)`` tokens."""
    device = prompt_ids.device
    b, s = prompt_ids.shape[0], prompt_ids.shape[-1]
    if s > max_seq_len:
        raise ValueError(f"prompt length {s} exceeds max_seq_len={max_seq_len}.")
    dtype = next(iter(model.embed.parameters())).dtype
    caches = [blk.attn.alloc_kv_cache(batch=b, max_seq=max_seq_len, device=device, dtype=dtype) for blk in model.blocks]
    x = _run_blocks(model, model.embed(prompt_ids), caches)
    logits = model.project_to_logits(model.final_norm(x)[:, -1:, :])
    out: list[Tensor] = []
    done = torch.zeros(b, dtype=torch.bool, device=device)
    for _ in range(max_new_tokens):
        tok = sample_logits(logits[:, -1, :], temperature, top_k, top_p)
        out.append(tok)
        if eos_token_id is not None:
            done |= tok.squeeze(-1) == eos_token_id
            if bool(done.all()):
                break
        x = _run_blocks(model, model.embed(tok), caches)
        logits = model.project_to_logits(model.final_norm(x))
    if not out:
        return prompt_ids
    return torch.cat([prompt_ids, *out], dim=-1)


def sample_logits(logits: Tensor, temperature: float, top_k: int, top_p: float) -> Tensor:
    """``(B, V)`` logits -> ``(B, 1)`` token ids."""
    if temperature == 0:
        return logits.argmax(dim=-1, keepdim=True)
    logits = logits.float() / temperature
    if top_k > 0:
        kth = logits.topk(min(top_k, logits.size(-1)), dim=-1).values[..., -1:]
        logits = logits.where(logits >= kth, torch.full_like(logits, -1e10))
    if top_p < 1.0:
        sl, si = logits.sort(dim=-1, descending=True)
        p = sl.softmax(dim=-1)
        sl = sl.masked_fill(p.cumsum(dim=-1) - p > top_p, -1e10)
        logits = torch.empty_like(logits).scatter_(-1, si, sl)
    return torch.multinomial(logits.softmax(dim=-1), num_samples=1)


_sample = sample_logits
