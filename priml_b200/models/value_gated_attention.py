"""Windowed attention with a value-embedding gate (``priml/model/value_gated_attention.py:46-305``).

Separate q/k/v projections; values may receive a per-layer value embedding
through ``2 * sigmoid(value_gate(x[..., :gate_channels]))`` (zero-initialized,
so the gate starts at 1); rotation by ``-theta`` at input precision
(``rotate_conjugate``), then per-head QK RMSNorm, then causal attention over a
window chosen per layer from an ``S`` / ``L`` pattern. The output projection is
zero-initialized. The attention kernel slot defaults to the fused kernel
(tcgen05 flash attention with a window on CUDA).
"""

from __future__ import annotations

from dataclasses import KW_ONLY, field
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable, PartialConfig
from priml_b200.models.attention import layer_window
from priml_b200.models.custom_types import ChannelsIn, propagate_attr
from priml_b200.models.init import InitFn, unit_fan_in_uniform
from priml_b200.models.linear import Linear
from priml_b200.models.norm import RMSNorm
from priml_b200.models.rope import rotate_conjugate

__all__ = ["ValueGatedAttention", "sdpa_attention"]


def sdpa_attention(q: Tensor, k: Tensor, v: Tensor, *, window: int) -> Tensor:
    """Causal attention admitting ``window`` keys of history (self included); ``[..., S, H, D]``."""
    from priml_b200.models.attention import SdpaFused

    w = -1 if window >= q.shape[-3] else window
    return SdpaFused()(q, k, v, is_causal=True, window=w)


class ValueGatedAttention(nn.Module):
    class Config(Fig["ValueGatedAttention"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        heads: int = -1
        channels_head: int = 128
        gate_channels: int = 32
        norm_qk: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        init_weight: InitFn = unit_fan_in_uniform
        kernel: Any = field(default_factory=lambda: PartialConfig(sdpa_attention))
        window: int = -1
        window_pattern: str = "SSSL"
        max_seq_len: int = -1
        gated: bool = True
        depth: int = -1

        def finalize(self):  # noqa: ANN201
            if self.channels_head <= 0 or self.channels_head % 2:
                raise ValueError(f"channels_head must be positive and even; got {self.channels_head}.")
            if self.heads == -1:
                if self.channels_in % self.channels_head:
                    raise ValueError("channels_in is not divisible by channels_head; set heads.")
                self.heads = self.channels_in // self.channels_head
            if self.window == -1 and self.max_seq_len > 0 and self.depth >= 0:
                self.window = layer_window(depth=self.depth, max_seq_len=self.max_seq_len, pattern=self.window_pattern)
            if self.gate_channels == -1:
                self.gate_channels = self.channels_in
            if not 0 < self.gate_channels <= self.channels_in:
                raise ValueError(f"gate_channels={self.gate_channels} must lie in (0, channels_in].")
            propagate_attr(self.norm_qk, "channels_in", self.channels_head, protocol=ChannelsIn)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if min(config.channels_in, config.heads, config.gate_channels) <= 0:
            raise ValueError("channels_in, heads and gate_channels must be positive.")
        self.config = config
        inner = config.heads * config.channels_head
        proj = Linear.Config(config.channels_in, inner, init_weight=config.init_weight)
        self.proj_q, self.proj_k, self.proj_v = (proj.copy_tree().make() for _ in range(3))
        self.proj_out = Linear.Config(inner, config.channels_in, init_weight=nn.init.zeros_).make()
        self.value_gate = (
            Linear.Config(config.gate_channels, config.heads, init_weight=nn.init.zeros_).make() if config.gated else None
        )
        self.norm_q = config.norm_qk.make()
        self.norm_k = config.norm_qk.make()
        self.attention = config.kernel.make()

    def reset_parameters(self) -> None:
        for m in (self.proj_q, self.proj_k, self.proj_v, self.proj_out):
            m.reset_parameters()
        if self.value_gate is not None:
            self.value_gate.reset_parameters()

    def forward(self, x: Tensor, *args: Any, cos_sin: tuple[Tensor, Tensor], value_embedding: Tensor | None = None,
                **kwargs: Any) -> Tensor:  # fmt: skip
        del args, kwargs
        c = self.config
        shape = (*x.shape[:-1], c.heads, c.channels_head)
        q, k, v = self.proj_q(x).view(shape), self.proj_k(x).view(shape), self.proj_v(x).view(shape)
        if value_embedding is not None:
            assert self.value_gate is not None, "a layer given a value embedding must be built gated"
            gate = 2 * torch.sigmoid(self.value_gate(x[..., : c.gate_channels]))
            v = v + gate.unsqueeze(-1) * value_embedding.view(shape)
        cos, sin = cos_sin
        q, k = rotate_conjugate(q, cos=cos, sin=sin), rotate_conjugate(k, cos=cos, sin=sin)
        q, k = self.norm_q(q), self.norm_k(k)
        window = c.window if c.window > 0 else q.shape[-3]
        return self.proj_out(self.attention(q, k, v, window=window).contiguous().flatten(-2))
