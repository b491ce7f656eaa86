"""Bounded, time-ordered key/value store for autoregressive decoding.

Counterpart of ``priml/model/kvcache.py:12-106``: the same public surface
(``alloc``, ``update``, ``freeze``, ``k`` / ``v`` as ``[..., H, max_seq, D]``
tensors whose first ``length`` rows are the visible keys, ``seen`` as the count
of every token ever appended so RoPE positions keep growing after eviction).

Storage is different. An allocated cache keeps ``2 * max_seq`` rows and a
moving window start. Appending past capacity only advances the start; the
visible rows are moved back to the front once the start reaches the slack, so
a decode loop at capacity copies about one row per token instead of shifting
the whole window on every token. Rows stay in time order, which is what a
bottom-right-aligned causal mask over a multi-token append needs.
"""

from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["KVCache"]


class KVCache:
    """Keys and values of the tokens seen so far, newest last, at most ``max_seq`` of them."""

    __slots__ = ("_kbuf", "_vbuf", "_start", "_window", "_read_only", "length", "seen")

    def __init__(self, k: Tensor, v: Tensor, length: int | None = None) -> None:
        """Wrap existing ``[..., H, S, D]`` tensors; their first ``length`` rows (default all) are visible.

        A wrapped cache has no slack rows: its capacity is ``S`` and eviction moves rows in place.
        """
        self._kbuf = k
        self._vbuf = v
        self._window = k.shape[-2]
        self._start = 0
        self._read_only = False
        self.length = self._window if length is None else int(length)
        if not 0 <= self.length <= self._window:
            raise ValueError(f"length {self.length} is outside [0, {self._window}].")
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
        """An empty cache of ``max_seq`` visible rows (MLA passes a separate value width)."""
        lead = (batch,) if isinstance(batch, int) else tuple(batch)
        width_v = channels_head if channels_v_head is None else channels_v_head
        rows = 2 * max_seq  # visible window + equal slack, so compaction never overlaps itself
        cache = cls.__new__(cls)
        cache._kbuf = torch.zeros((*lead, heads, rows, channels_head), device=device, dtype=dtype)
        cache._vbuf = torch.zeros((*lead, heads, rows, width_v), device=device, dtype=dtype)
        cache._window = max_seq
        cache._start = 0
        cache._read_only = False
        cache.length = 0
        cache.seen = 0
        return cache

    # ------------------------------------------------------------------ views
    @property
    def max_seq(self) -> int:
        return self._window

    @property
    def k(self) -> Tensor:
        """``[..., H, max_seq, D]`` view; rows ``[0, length)`` hold the visible keys, oldest first."""
        return self._kbuf.narrow(-2, self._start, self._window)

    @property
    def v(self) -> Tensor:
        return self._vbuf.narrow(-2, self._start, self._window)

    def visible(self) -> tuple[Tensor, Tensor]:
        return self._kbuf.narrow(-2, self._start, self.length), self._vbuf.narrow(-2, self._start, self.length)

    # ------------------------------------------------------------------ writes
    def freeze(self) -> KVCache:
        """A cache over the same storage whose ``update`` appends nothing (re-scoring one prefix)."""
        other = KVCache.__new__(KVCache)
        for name in KVCache.__slots__:
            setattr(other, name, getattr(self, name))
        other._read_only = True
        return other

    def update(self, k: Tensor, v: Tensor) -> tuple[Tensor, Tensor]:
        """Append ``[..., H, s, D]`` rows, evicting the oldest beyond ``max_seq``; returns the visible rows."""
        if self._read_only:
            return self.visible()
        s = k.shape[-2]
        if s > self._window:
            raise ValueError(f"cannot append {s} rows to a cache of {self._window} rows.")
        evict = max(0, self.length + s - self._window)
        keep = self.length - evict
        start = self._start + evict
        slack = self._kbuf.shape[-2] - self._window
        if start + keep + s > self._kbuf.shape[-2] or start > slack:
            # Move the surviving rows to the front. With slack >= max_seq the source lies past the
            # destination; a wrapped cache (no slack) may overlap, so its rows go through a copy.
            src_k = self._kbuf.narrow(-2, start, keep)
            src_v = self._vbuf.narrow(-2, start, keep)
            if start < keep:
                src_k, src_v = src_k.clone(), src_v.clone()
            self._kbuf.narrow(-2, 0, keep).copy_(src_k)
            self._vbuf.narrow(-2, 0, keep).copy_(src_v)
            start = 0
        self._kbuf.narrow(-2, start + keep, s).copy_(k)
        self._vbuf.narrow(-2, start + keep, s).copy_(v)
        self._start = start
        self.length = keep + s
        self.seen += s
        return self.visible()
