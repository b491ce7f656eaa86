"""Token embeddings (``priml/model/embedding.py:18-80``, ``priml/model/narrow_embedding.py:38-93``)."""

from __future__ import annotations

from dataclasses import KW_ONLY, field
from functools import partial
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsOut, ShardStyle, propagate_attr
from priml_b200.models.init import InitFn, call_init, truncated_normal

__all__ = ["Embedding", "NarrowEmbedding"]


class Embedding(nn.Embedding):
    """Embedding table drawn by ``init_weight`` (truncated normal, std 0.02)."""

    class Config(Fig["Embedding"], kw_only=False):
        channels_out: int = -1
        _: KW_ONLY
        num_embeddings: int = -1
        padding_idx: int | None = None
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None
        shard: ShardStyle | None = None
        depth: int = -1
        init_weight: InitFn = partial(truncated_normal, std=0.02)

    def __init__(self, config: Config) -> None:
        self.shard = config.shard
        self.depth = config.depth
        self._init_weight = config.init_weight
        super().__init__(
            num_embeddings=config.num_embeddings,
            embedding_dim=config.channels_out,
            padding_idx=config.padding_idx,
            device=config.device,
            dtype=config.dtype,
        )

    def reset_parameters(self) -> None:
        if not hasattr(self, "_init_weight"):
            return super().reset_parameters()
        call_init(self._init_weight, self.weight, depth=self.depth)
        if self.padding_idx is not None:
            with torch.no_grad():
                self.weight[self.padding_idx].fill_(0)
        return None

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        if input.is_cuda and torch.is_autocast_enabled("cuda"):
            # Gather straight into the compute dtype: the table row is read once
            # and written once at bf16 width.
            return nn.functional.embedding(input, self.weight).to(torch.get_autocast_dtype("cuda"))
        return super().forward(input)


class NarrowEmbedding(nn.Module):
    """A table drawn at full precision by ``inner`` and then held at ``dtype``.

    Drawing straight into bf16 would quantize every draw and change the spread;
    this module owns both steps so the cast always follows the draw
    (``priml/model/narrow_embedding.py:38-93``).
    """

    class Config(Fig["NarrowEmbedding"], kw_only=False):
        dtype: torch.dtype | None = None
        """Width the table is held at; ``None`` keeps ``inner``'s."""
        _: KW_ONLY
        inner: Makeable[nn.Module] = field(default_factory=Embedding.Config)
        channels_out: int = -1
        num_embeddings: int = -1

        def finalize(self):  # noqa: ANN201
            propagate_attr(self.inner, "channels_out", self.channels_out, protocol=ChannelsOut)
            propagate_attr(self.inner, "num_embeddings", self.num_embeddings)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.dtype = config.dtype
        self.inner = config.inner.make()
        self._narrow()

    @property
    def weight(self) -> Tensor:
        return self.inner.weight

    def reset_parameters(self) -> None:
        if self.dtype is not None:
            self.inner.to(dtype=torch.float32)
        self.inner.reset_parameters()
        self._narrow()

    def _narrow(self) -> None:
        if self.dtype is not None:
            self.inner.to(dtype=self.dtype)

    def forward(self, tokens: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        return self.inner(tokens)
