"""Tokens prepended to a puzzle grid (``priml/baselines/sudoku/prefix.py:1-296``).

A prefix module is called as ``prefix(batch_size, **batch_kwargs) -> [B, P, C]``
and declares ``num_tokens`` so the model can size its latent state.

* :class:`RegisterTokens` -- ``P`` learned (or frozen random) tokens shared by
  every example; the halt readout at position 0 then reads a dedicated token.
* :class:`SparsePuzzleEmbedding` -- a per-puzzle vector (one row per puzzle
  identifier) reshaped into ``num_tokens`` tokens. The full table is a BUFFER:
  only the batch's rows are copied into a preallocated ``local_weights`` leaf
  that receives gradients, and ``local_ids`` records which rows they were. A
  sparse optimizer (``SignSGD`` with a ``sparse_embedding`` group) scatters the
  update back, so a table of a million puzzles costs no dense gradient or
  optimizer state.
* :class:`PrefixStack` -- concatenates several prefix modules along the tokens.
"""

from __future__ import annotations

import math
from dataclasses import field
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.baselines.sudoku.embedding import HasHiddenSize
from priml_b200.config import Fig, Makeable
from priml_b200.models.init import truncated_normal

__all__ = ["PrefixStack", "RegisterTokens", "SparsePuzzleEmbedding"]


def _scale(hidden_size: int, embed_scale: float) -> float:
    return math.sqrt(hidden_size) if embed_scale < 0 else embed_scale


class RegisterTokens(nn.Module):
    class Config(Fig["RegisterTokens"]):
        num_tokens: int = 1
        hidden_size: int = -1
        init_std: float = 1.0
        learnable: bool = True
        embed_scale: float = -1.0

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.hidden_size <= 0:
            raise ValueError(f"hidden_size must be positive; got {config.hidden_size} (inherited from the model).")
        self.config = config
        self.embed_scale = _scale(config.hidden_size, config.embed_scale)
        t = torch.empty(config.num_tokens, config.hidden_size)
        truncated_normal(t, std=config.init_std / self.embed_scale, depth=-1, variance_correction=True)
        if config.learnable:
            self.register_tokens = nn.Parameter(t)
        else:
            self.register_tokens = nn.Buffer(t, persistent=True)

    def forward(self, batch_size: int, **kwargs: Any) -> Tensor:
        del kwargs
        return self.embed_scale * self.register_tokens.unsqueeze(0).expand(batch_size, -1, -1)


class SparsePuzzleEmbedding(nn.Module):
    class Config(Fig["SparsePuzzleEmbedding"]):
        num_puzzles: int = 1
        num_tokens: int = 16
        channels: int = -1
        """Per-puzzle vector width; -1 uses ``hidden_size``. Narrower vectors are zero-padded."""
        hidden_size: int = -1
        batch_size: int = 384
        """Rows of the preallocated gradient leaf (the training batch size)."""
        init_std: float = 0.0
        embed_scale: float = -1.0
        dtype: torch.dtype | None = None

        def finalize(self):  # noqa: ANN201
            if self.channels == -1:
                self.channels = self.hidden_size
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.hidden_size <= 0 or config.channels <= 0:
            raise ValueError(
                f"hidden_size and channels must be positive; got {config.hidden_size} and {config.channels}."
            )
        if config.num_puzzles < 1:
            raise ValueError(f"num_puzzles must be positive; got {config.num_puzzles}.")
        if config.channels > config.num_tokens * config.hidden_size:
            raise ValueError(f"channels {config.channels} exceed num_tokens * hidden_size.")
        self.config = config
        self.embed_scale = _scale(config.hidden_size, config.embed_scale)
        table = torch.zeros(config.num_puzzles, config.channels)
        if config.init_std > 0:
            truncated_normal(table, std=config.init_std, depth=-1, variance_correction=True)
        self.weights = nn.Buffer(table, persistent=True)
        self.local_weights = nn.Buffer(torch.zeros(config.batch_size, config.channels, requires_grad=True),
                                       persistent=False)  # fmt: skip
        self.local_ids = nn.Buffer(torch.zeros(config.batch_size, dtype=torch.int32), persistent=False)

    def forward(self, batch_size: int, **kwargs: Any) -> Tensor:
        ids = kwargs.get("puzzle_identifiers")
        if not isinstance(ids, Tensor):
            raise TypeError(f"SparsePuzzleEmbedding needs puzzle_identifiers in the batch; got {type(ids).__name__}.")
        vec = self._lookup(ids)
        c = self.config
        width = c.num_tokens * c.hidden_size
        if vec.shape[-1] < width:
            vec = nn.functional.pad(vec, (0, width - vec.shape[-1]))
        return self.embed_scale * vec.reshape(batch_size, c.num_tokens, c.hidden_size)

    def _lookup(self, ids: Tensor) -> Tensor:
        dtype = self.config.dtype
        if not self.training:
            rows = self.weights[ids.long()]
            return rows if dtype is None else rows.to(dtype)
        if ids.shape[0] != self.local_ids.shape[0]:
            raise ValueError(f"the gradient leaf holds {self.local_ids.shape[0]} rows; got a batch of {ids.shape[0]}.")
        with torch.no_grad():
            self.local_weights.copy_(self.weights[ids.long()])
            self.local_ids.copy_(ids.to(torch.int32))
        return self.local_weights if dtype is None else self.local_weights.to(dtype)

    def _apply(self, fn: Any, recurse: bool = True) -> SparsePuzzleEmbedding:
        out = super()._apply(fn, recurse=recurse)
        # ``.to()`` produces non-leaf copies; restore the gradient leaf on the new device
        self.local_weights = nn.Buffer(self.local_weights.detach().requires_grad_(True), persistent=False)
        self.local_ids = nn.Buffer(self.local_ids.detach(), persistent=False)
        return out


class PrefixStack(nn.Module):
    class Config(Fig["PrefixStack"]):
        parts: list[Makeable[nn.Module]] = field(default_factory=list)
        hidden_size: int = -1

        def finalize(self):  # noqa: ANN201
            for p in self.parts:
                if isinstance(p, HasHiddenSize) and p.hidden_size == -1:
                    p.hidden_size = self.hidden_size
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.parts = nn.ModuleList(p.make() for p in config.parts)

    def forward(self, batch_size: int, **kwargs: Any) -> Tensor:
        return torch.cat([p(batch_size, **kwargs) for p in self.parts], dim=1)
