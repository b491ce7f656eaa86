"""Grid-puzzle input embedding (``priml/baselines/sudoku/embedding.py:1-352``).

The input is ``embed_scale * table[token]`` with ``embed_scale = sqrt(C)`` and
the table drawn at ``std = 1 / sqrt(C)`` (the rescale trick: tables live at the
scale an optimizer steps well, activations enter at unit scale). Additive
channels are summed on top IN CONFIG ORDER -- the order is part of the numerics
because floating-point addition does not associate:

* :class:`FactoredPositions` -- learned row, column and box tables, indexed by
  the cell each flat position maps to (81 cells -> 9 + 9 + 9 rows instead of 81);
* :class:`PredictionFeedback` -- a table over the previous step's decoded grid,
  zero at init so a fresh recurrent model starts as its plain counterpart.

Every table is an ``[N, C]`` parameter; lookups are gathers (no one-hot GEMM).
"""

from __future__ import annotations

import math
from dataclasses import field
from typing import Any, Protocol, runtime_checkable

import torch
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable
from priml_b200.models.embedding import Embedding
from priml_b200.models.init import truncated_normal

__all__ = [
    "FactoredPositions",
    "GridChannel",
    "GridEmbedding",
    "HasGridLen",
    "HasHiddenSize",
    "HasVocabSize",
    "PredictionFeedback",
]


@runtime_checkable
class GridChannel(Protocol):
    """``channel(tokens [B, L], embeddings [B, L, C]) -> [B?, L, C]`` (or an empty tensor to add nothing)."""

    def __call__(self, tokens: Tensor, embeddings: Tensor) -> Tensor: ...


@runtime_checkable
class HasHiddenSize(Protocol):
    hidden_size: int


@runtime_checkable
class HasGridLen(Protocol):
    grid_len: int


@runtime_checkable
class HasVocabSize(Protocol):
    vocab_size: int


def _scale(hidden_size: int, embed_scale: float) -> float:
    return math.sqrt(hidden_size) if embed_scale < 0 else embed_scale


def _table(rows: int, hidden_size: int, init_std: float) -> nn.Parameter:
    """``[rows, C]`` table with realized std ``init_std / sqrt(C)`` (zeros when ``init_std == 0``)."""
    w = torch.zeros(rows, hidden_size)
    if init_std > 0:
        truncated_normal(w, std=init_std / math.sqrt(hidden_size), depth=-1, variance_correction=True)
    return nn.Parameter(w)


class FactoredPositions(nn.Module):
    """Row + column + box position tables for a ``grid_shape`` grid tiled by ``box_shape`` boxes."""

    class Config(Fig["FactoredPositions"]):
        grid_shape: tuple[int, int] = (9, 9)
        box_shape: tuple[int, int] = (3, 3)
        hidden_size: int = -1
        init_std: float = 1.0
        embed_scale: float = -1.0
        """Runtime multiplier; -1 uses ``sqrt(hidden_size)``, matching the token embedding."""

    def __init__(self, config: Config) -> None:
        super().__init__()
        rows, cols = config.grid_shape
        br, bc = config.box_shape
        if rows % br or cols % bc:
            raise ValueError(f"box_shape {config.box_shape} does not tile grid_shape {config.grid_shape}.")
        if config.hidden_size <= 0:
            raise ValueError(f"hidden_size must be positive; got {config.hidden_size} (inherited from the model).")
        self.config = config
        self.embed_scale = _scale(config.hidden_size, config.embed_scale)
        cell = torch.arange(rows * cols)
        r, c = cell // cols, cell % cols
        self.row_index = nn.Buffer(r, persistent=False)
        self.col_index = nn.Buffer(c, persistent=False)
        self.box_index = nn.Buffer((r // br) * (cols // bc) + c // bc, persistent=False)
        n_boxes = (rows // br) * (cols // bc)
        self.embed_pos_row = _table(rows, config.hidden_size, config.init_std)
        self.embed_pos_col = _table(cols, config.hidden_size, config.init_std)
        self.embed_pos_box = _table(n_boxes, config.hidden_size, config.init_std)

    def forward(self, tokens: Tensor, embeddings: Tensor) -> Tensor:
        del tokens
        pos = self.embed_pos_row[self.row_index] + self.embed_pos_col[self.col_index] + self.embed_pos_box[self.box_index]
        return self.embed_scale * pos.to(embeddings.dtype)


class PredictionFeedback(nn.Module):
    """Embeds the grid the previous recurrent step decoded; set through :meth:`set_feedback`.

    The ids are consumed by the next forward (one-shot), so a stale grid can
    never leak into a later call; with none set the channel adds nothing.
    """

    class Config(Fig["PredictionFeedback"]):
        vocab_size: int = -1
        hidden_size: int = -1
        init_std: float = 0.0
        embed_scale: float = -1.0

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.hidden_size <= 0 or config.vocab_size <= 0:
            raise ValueError(
                f"vocab_size and hidden_size must be positive; got {config.vocab_size} and {config.hidden_size}."
            )
        self.config = config
        self.embed_scale = _scale(config.hidden_size, config.embed_scale)
        self.embed_feedback = _table(config.vocab_size, config.hidden_size, config.init_std)
        self._ids: Tensor | None = None

    def set_feedback(self, feedback_ids: Tensor | None) -> None:
        self._ids = feedback_ids

    def forward(self, tokens: Tensor, embeddings: Tensor) -> Tensor:
        del tokens
        ids, self._ids = self._ids, None
        if ids is None:
            return embeddings.new_empty(0)
        return self.embed_scale * self.embed_feedback[ids].to(embeddings.dtype)


class GridEmbedding(nn.Module):
    """Token embedding of a puzzle grid plus additive channels."""

    class Config(Fig["GridEmbedding"]):
        vocab_size: int = 11
        hidden_size: int = -1
        grid_shape: tuple[int, ...] = (81,)
        channels: list[Makeable[Any]] = field(default_factory=list)
        """Additive channels, summed in this order."""

        @property
        def grid_len(self) -> int:
            return math.prod(self.grid_shape)

        def finalize(self):  # noqa: ANN201
            for ch in self.channels:
                if isinstance(ch, HasHiddenSize) and ch.hidden_size == -1:
                    ch.hidden_size = self.hidden_size
                if isinstance(ch, HasGridLen) and ch.grid_len == -1:
                    ch.grid_len = self.grid_len
                if isinstance(ch, HasVocabSize) and ch.vocab_size == -1:
                    ch.vocab_size = self.vocab_size
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.hidden_size <= 0:
            raise ValueError(f"hidden_size must be positive; got {config.hidden_size} (inherited from the model).")
        self.config = config
        self.embed_scale = math.sqrt(config.hidden_size)
        self.embed_tokens = Embedding.Config(channels_out=config.hidden_size, num_embeddings=config.vocab_size).make()
        truncated_normal(self.embed_tokens.weight.data, std=1.0 / self.embed_scale, depth=-1, variance_correction=True)
        self.channels = nn.ModuleList(c.make() for c in config.channels)

    def forward(self, tokens: Tensor) -> Tensor:
        x = self.embed_scale * self.embed_tokens(tokens)
        for ch in self.channels:
            add = ch(tokens, x)
            if add.numel():
                x = x + add
        return x
