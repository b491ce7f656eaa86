"""Static KV cache with FIFO eviction (``priml/model/kvcache.py:12-106``).

Layout ``[..., H, max_seq, D]``; ``length`` is the valid prefix (capped at
``max_seq``), ``seen`` counts every token ever written so RoPE positions keep
increasing after eviction.
"""

from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["KVCache"]


class KVCache:
    __slots__ = ("k", "length", "seen", "v")

    def __init__(self, k: Tensor, v: Tensor, length: int | None = None) -> None:
        self.k = k
        self.v = v
        self.length = k.shape[-2] if length is None else length
        self.seen = self.length

    @classmethod
    def alloc(
        cls,
        *,
        batch: int | tuple[int, ...],
        heads: int,
        max_seq: int,
        channels_head: int,
        channels_v_head: int | None = None,
        device: torch.device | str | None = None,
        dtype: torch.dtype | None = None,
    ) -> KVCache:
        if isinstance(batch, int):
            batch = (batch,)
        dv = channels_head if channels_v_head is None else channels_v_head
        k = torch.zeros((*batch, heads, max_seq, channels_head), device=device, dtype=dtype)
        v = torch.zeros((*batch, heads, max_seq, dv), device=device, dtype=dtype)
        return cls(k, v, length=0)

    @property
    def max_seq(self) -> int:
        return self.k.shape[-2]

    def freeze(self) -> KVCache:
        frozen = _FrozenKVCache(self.k, self.v, self.length)
        frozen.seen = self.seen
        return frozen

    def update(self, k: Tensor, v: Tensor) -> tuple[Tensor, Tensor]:
        s = k.shape[-2]
        if s > self.max_seq:
            raise ValueError(f"Update length {s} exceeds cache capacity {self.max_seq}.")
        overflow = self.length + s - self.max_seq
        if overflow > 0:
            keep = self.length - overflow
            self.k[..., :keep, :] = self.k[..., overflow : self.length, :].clone()
            self.v[..., :keep, :] = self.v[..., overflow : self.length, :].clone()
            self.length = keep
        end = self.length + s
        self.k[..., self.length : end, :] = k
        self.v[..., self.length : end, :] = v
        self.length = end
        self.seen += s
        return self.k[..., :end, :], self.v[..., :end, :]


class _FrozenKVCache(KVCache):
    """Cache whose ``update`` is a no-op (repeated passes over one prefix)."""

    def update(self, k: Tensor, v: Tensor) -> tuple[Tensor, Tensor]:
        del k, v
        return self.k[..., : self.length, :], self.v[..., : self.length, :]
