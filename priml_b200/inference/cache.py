"""Static KV caches for batched decoding: fixed buffers, per-sequence lengths on the device.

:class:`priml_b200.models.kvcache.KVCache` (the reference's cache,
``priml/model/kvcache.py:12-106``) keeps its fill level as a Python int, so every
step depends on host state and cannot be replayed from a CUDA graph. The caches
here keep that state on the device instead:

* one :class:`CacheState` per decoder holds ``lengths`` (int32 ``[B]``): the number
  of tokens each sequence has in the cache. All layers share it; the decoder
  advances it once per forward, after the last layer.
* one :class:`StaticKVCache` per attention layer holds ``[B, Hkv, T, D]`` key and
  value buffers that never move or grow.

A layer hands its new keys to :meth:`StaticKVCache.attend`, which writes them at
rows ``lengths[b] + i`` and attends over the visible rows:

* one new token per sequence (decode): the decode kernel, which reads the lengths
  on the device;
* a prompt into empty rows (prefill): causal flash attention over the new keys only;
* anything else (a chunk appended to a partly filled cache): SDPA over the buffer
  with a per-sequence mask.

Rows past ``T`` are not written (the index is clamped to the last row); the
decoder tracks lengths on the host as well and refuses to overflow.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200 import ops

__all__ = ["CacheState", "StaticKVCache"]


@dataclass
class CacheState:
    """Per-sequence fill levels shared by every layer's cache."""

    lengths: Tensor  # int32 [B], on the cache's device
    capacity: int
    fresh: bool = False  # set while prefilling rows that are all empty: attend over the new keys only

    @classmethod
    def create(cls, batch: int, capacity: int, device: torch.device | str | None = None) -> CacheState:
        return cls(torch.zeros(batch, dtype=torch.int32, device=device), capacity)

    def positions(self, s: int) -> Tensor:
        """``[B, s, 1]`` RoPE positions of ``s`` tokens appended to every sequence."""
        return (self.lengths[:, None] + torch.arange(s, device=self.lengths.device, dtype=torch.int32))[..., None]

    def advance(self, s: int) -> None:
        self.lengths.add_(s)

    def select(self, rows: slice) -> CacheState:
        """The state of a contiguous range of sequences (a view: advancing it advances these rows)."""
        return CacheState(self.lengths[rows], self.capacity, self.fresh)


class StaticKVCache:
    """Fixed ``[B, Hkv, T, D]`` key/value buffers of one attention layer."""

    __slots__ = ("k", "v", "state")

    def __init__(self, k: Tensor, v: Tensor, state: CacheState) -> None:
        self.k, self.v, self.state = k, v, state

    @classmethod
    def alloc(
        cls,
        state: CacheState,
        *,
        heads: int,
        channels_head: int,
        channels_v_head: int | None = None,
        device: torch.device | str | None = None,
        dtype: torch.dtype | None = None,
    ) -> StaticKVCache:
        b, t = state.lengths.shape[0], state.capacity
        k = torch.zeros(b, heads, t, channels_head, device=device, dtype=dtype)
        v = torch.zeros(b, heads, t, channels_v_head or channels_head, device=device, dtype=dtype)
        return cls(k, v, state)

    def select(self, rows: slice, state: CacheState) -> StaticKVCache:
        return StaticKVCache(self.k[rows], self.v[rows], state)

    @property
    def seen(self) -> int:
        raise RuntimeError("a static cache keeps its lengths on the device; pass positions explicitly")

    # ------------------------------------------------------------------ write + attend
    def _write(self, k: Tensor, v: Tensor) -> None:
        b, s = k.shape[0], k.shape[1]
        t = self.k.shape[2]
        rows = (self.state.lengths[:, None].long() + torch.arange(s, device=k.device)).clamp_(max=t - 1)
        bidx = torch.arange(b, device=k.device)[:, None]
        self.k.transpose(1, 2)[bidx, rows] = k.to(self.k.dtype)
        self.v.transpose(1, 2)[bidx, rows] = v.to(self.v.dtype)

    def attend(self, q: Tensor, k: Tensor, v: Tensor, *, scale: float | None = None, window: int = -1) -> Tensor:
        """Append ``[B, s, Hkv, D]`` keys/values and attend ``[B, s, H, D]`` queries; returns ``[B, s, H, Dv]``."""
        win = None if window is None or window < 0 else int(window)
        self._write(k, v)
        s = q.shape[1]
        if s == 1:
            out = ops.decode_attention(q[:, 0], self.k, self.v, self.state.lengths + 1, scale=scale, window=win)
            return out[:, None]
        if self.state.fresh:
            return ops.attention(q, k, v, causal=True, scale=scale, window=win)
        return self._attend_masked(q, scale, win)

    def _attend_masked(self, q: Tensor, scale: float | None, window: int | None) -> Tensor:
        b, s, h, _ = q.shape
        hkv, t = self.k.shape[1], self.k.shape[2]
        qpos = self.state.lengths[:, None].long() + torch.arange(s, device=q.device)  # [B, s]
        kpos = torch.arange(t, device=q.device)
        ok = kpos[None, None, :] <= qpos[:, :, None]
        if window is not None:
            ok &= kpos[None, None, :] >= qpos[:, :, None] - window
        kf = self.k.repeat_interleave(h // hkv, dim=1)
        vf = self.v.repeat_interleave(h // hkv, dim=1)
        out = F.scaled_dot_product_attention(q.transpose(1, 2), kf.to(q.dtype), vf.to(q.dtype), attn_mask=ok[:, None],
                                             scale=scale)  # fmt: skip
        return out.transpose(1, 2)
