"""Residual transformer block (``priml/model/transformer.py:29-178``).

Submodule names ``attn``, ``ffn``, ``norm1``, ``norm2`` match the reference so
state dicts interchange. ``checkpoint=True`` recomputes the block in backward.
"""

from __future__ import annotations

from dataclasses import KW_ONLY, field
from typing import Any

import torch
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint as torch_checkpoint

from priml_b200.config import Fig, Makeable
from priml_b200.models.attention import SelfAttention
from priml_b200.models.custom_types import (
    ChannelsIn,
    ChannelsOut,
    HasDepth,
    HeadGeometry,
    ShardableConfig,
    propagate_attr,
)
from priml_b200.models.norm import RMSNorm
from priml_b200.models.swiglu import SwiGLU

__all__ = ["TransformerBlock"]


class TransformerBlock(nn.Module):
    class Config(Fig["TransformerBlock"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        attn: Makeable[nn.Module] = field(default_factory=SelfAttention.Config)
        ffn: Makeable[nn.Module] = field(default_factory=SwiGLU.Config)
        norm1: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        norm2: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        prenorm: bool = True
        checkpoint: bool = False
        depth: int = -1

        @property
        def channels_out(self) -> int:
            return self.channels_in

        @property
        def heads(self) -> int:
            return self.attn.heads if isinstance(self.attn, HeadGeometry) else 1

        @property
        def channels_head(self) -> int:
            return self.attn.channels_head if isinstance(self.attn, HeadGeometry) else self.channels_in

        def finalize(self):  # noqa: ANN201
            for cfg in (self.attn, self.ffn, self.norm1, self.norm2):
                propagate_attr(cfg, "channels_in", self.channels_in, protocol=ChannelsIn)
                propagate_attr(cfg, "channels_out", self.channels_in, protocol=ChannelsOut)
                propagate_attr(cfg, "depth", self.depth, protocol=HasDepth)
            if isinstance(self.ffn, ShardableConfig):
                self.ffn.shard = "colwise"
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.prenorm = config.prenorm
        self.checkpoint = config.checkpoint
        self.depth = config.depth
        self.attn = config.attn.make()
        self.ffn = config.ffn.make()
        self.norm1 = config.norm1.make()
        self.norm2 = config.norm2.make()

    def reset_parameters(self) -> None:
        for m in (self.attn, self.ffn, self.norm1, self.norm2):
            if hasattr(m, "reset_parameters"):
                m.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Any:
        if self.checkpoint and torch.is_grad_enabled():
            return torch_checkpoint(self._forward, x, *args, use_reentrant=False, **kwargs)
        return self._forward(x, *args, **kwargs)

    @staticmethod
    def _unpack(res: Any) -> tuple[Tensor, Any]:
        if isinstance(res, Tensor):
            return res, None
        return res[0], res[1]

    def _forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Any:
        if self.prenorm:
            a, cache = self._unpack(self.attn(self.norm1(x), *args, **kwargs))
            x = x + a
            x = x + self.ffn(self.norm2(x))
        else:
            a, cache = self._unpack(self.attn(x, *args, **kwargs))
            x = self.norm1(x + a)
            x = self.norm2(x + self.ffn(x))
        if "cache" in kwargs and cache is not None:
            return x, cache
        return x
