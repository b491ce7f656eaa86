"""Token sampling that stays on the device.

:func:`priml_b200.models.generate.sample_logits` follows the reference
(``priml/model/generate.py:131-188``): one temperature / top-k / top-p for the
batch, ``torch.multinomial`` for the draw. A server batches requests with
different settings and wants the draw inside the decode step's CUDA graph, so
here:

* the settings are per-row device tensors (:class:`SamplingParams` builds them);
* the draw is Gumbel-max -- ``argmax(z + g)`` with ``g = -log(-log(u))`` -- which
  samples ``softmax(z)`` exactly, from one ``rand`` and one reduction, with
  static shapes and no host synchronisation;
* top-k and top-p need each row sorted once; when no row uses either,
  ``filtered=False`` skips the sort.

The filtering order is the reference's (HF's): temperature, then top-k, then top-p
on the exclusive cumulative mass of what top-k kept. Temperature 0 is greedy.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

__all__ = ["SamplingParams", "sample"]


@dataclass(frozen=True)
class SamplingParams:
    """One request's sampling settings."""

    temperature: float = 1.0
    top_k: int = 0  # 0: no top-k
    top_p: float = 1.0  # 1: no top-p

    @property
    def filtered(self) -> bool:
        return self.temperature > 0 and (self.top_k > 0 or self.top_p < 1.0)

    @staticmethod
    def stack(params: list[SamplingParams], device: torch.device | str | None = None) -> tuple[Tensor, Tensor, Tensor]:
        """Per-row ``(temperature f32, top_k i64, top_p f32)`` tensors."""
        t = torch.tensor([p.temperature for p in params], dtype=torch.float32, device=device)
        k = torch.tensor([p.top_k for p in params], dtype=torch.int64, device=device)
        p_ = torch.tensor([p.top_p for p in params], dtype=torch.float32, device=device)
        return t, k, p_


def _gumbel(shape: torch.Size, device: torch.device, generator: torch.Generator | None) -> Tensor:
    u = torch.rand(shape, device=device, generator=generator)
    u = u.clamp_(min=torch.finfo(torch.float32).tiny, max=1.0 - torch.finfo(torch.float32).eps)
    return -torch.log(-torch.log(u))


def sample(
    logits: Tensor,
    temperature: Tensor,
    top_k: Tensor,
    top_p: Tensor,
    *,
    filtered: bool = True,
    generator: torch.Generator | None = None,
) -> Tensor:
    """``[B, V]`` logits and per-row settings ``[B]`` -> ``[B]`` int64 token ids."""
    greedy = logits.argmax(dim=-1)
    z = logits.float() / temperature.clamp_min(1e-6)[:, None]
    if not filtered:
        drawn = (z + _gumbel(z.shape, z.device, generator)).argmax(dim=-1)
        return torch.where(temperature > 0, drawn, greedy)
    sz, si = z.sort(dim=-1, descending=True)
    rank = torch.arange(z.shape[-1], device=z.device)
    keep = (top_k[:, None] <= 0) | (rank[None, :] < top_k[:, None])
    sz = sz.masked_fill(~keep, float("-inf"))
    prob = sz.softmax(dim=-1)
    keep &= (prob.cumsum(dim=-1) - prob) <= top_p[:, None]
    sz = sz.masked_fill(~keep, float("-inf"))
    pick = (sz + _gumbel(sz.shape, sz.device, generator)).argmax(dim=-1, keepdim=True)
    drawn = si.gather(-1, pick).squeeze(-1)
    return torch.where(temperature > 0, drawn, greedy)
