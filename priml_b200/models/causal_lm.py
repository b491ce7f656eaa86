"""Decoder-only language model (``priml/model/causal_lm.py:45-176``).

``embed -> blocks -> final_norm -> lm_head`` with the reference's module names
(``embed.weight``, ``blocks.{i}.*``, ``final_norm.weight``, ``lm_head.weight``).

``forward`` returns logits like the reference. Training goes through
:meth:`CausalLM.token_loss`, which never materializes the ``[tokens, vocab]``
logits: on CUDA it runs the chunked fused linear + cross-entropy kernel.
"""

from __future__ import annotations

from copy import deepcopy
from dataclasses import KW_ONLY, field
from typing import Any

from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, propagate_attr
from priml_b200.models.embedding import Embedding
from priml_b200.models.linear import Linear
from priml_b200.models.norm import RMSNorm
from priml_b200.models.transformer import TransformerBlock, add_then_norm

__all__ = ["CausalLM"]


class CausalLM(nn.Module):
    class Config(Fig["CausalLM"], kw_only=False):
        vocab_size: int = -1
        _: KW_ONLY
        channels: int = -1
        num_layers: int = -1
        block: Any = field(default_factory=TransformerBlock.Config)
        """One block config broadcast ``num_layers`` times (each copy gets its
        ``depth``), or an explicit per-layer list."""
        final_norm: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        tie_embeddings: bool = False
        lm_head: Makeable[nn.Module] | None = None
        embed: Makeable[nn.Module] | None = None
        """Token table; ``None`` builds ``Embedding`` (truncated normal 0.02)."""

        def finalize(self):  # noqa: ANN201
            if self.vocab_size < 1:
                raise ValueError(f"vocab_size must be > 0, got {self.vocab_size}.")
            if self.num_layers < 1:
                raise ValueError(f"num_layers must be > 0, got {self.num_layers}.")
            if self.channels < 1:
                raise ValueError(f"channels must be > 0, got {self.channels}.")
            if isinstance(self.block, list) and len(self.block) != self.num_layers:
                raise ValueError(f"block list length {len(self.block)} != num_layers={self.num_layers}.")
            blocks = self.block if isinstance(self.block, list) else [self.block]
            for cfg in (*blocks, self.final_norm):
                propagate_attr(cfg, "channels_in", self.channels, protocol=ChannelsIn)
            if self.lm_head is not None:
                propagate_attr(self.lm_head, "channels_in", self.channels, protocol=ChannelsIn)
                propagate_attr(self.lm_head, "channels_out", self.vocab_size, protocol=ChannelsOut)
            if self.embed is not None:
                propagate_attr(self.embed, "channels_out", self.channels, protocol=ChannelsOut)
                propagate_attr(self.embed, "num_embeddings", self.vocab_size)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.vocab_size = config.vocab_size
        self.channels = config.channels
        self.num_layers = config.num_layers
        self.tie_embeddings = config.tie_embeddings
        if config.embed is not None:
            self.embed = config.embed.make()
        else:
            self.embed = Embedding.Config(
                channels_out=config.channels, num_embeddings=config.vocab_size, shard="vocab"
            ).make()
        templates = config.block if isinstance(config.block, list) else [config.block]
        self.blocks = nn.ModuleList()
        for i in range(config.num_layers):
            cfg = deepcopy(templates[i] if isinstance(config.block, list) else templates[0])
            if hasattr(cfg, "depth"):
                object.__setattr__(cfg, "depth", i)
            self.blocks.append(cfg.make())
        self.final_norm = config.final_norm.make()
        if config.tie_embeddings:
            self.lm_head: nn.Module | None = None
        elif config.lm_head is not None:
            self.lm_head = config.lm_head.make()
        else:
            self.lm_head = Linear.Config(
                channels_in=config.channels, channels_out=config.vocab_size, bias=False, shard="vocab"
            ).make()

    def reset_parameters(self) -> None:
        for m in (self.embed, self.final_norm, *self.blocks, self.lm_head):
            if m is not None and hasattr(m, "reset_parameters"):
                m.reset_parameters()

    @property
    def output_weight(self) -> Tensor:
        """The ``[vocab, channels]`` matrix that maps hidden states to logits."""
        if self.tie_embeddings:
            return self.embed.weight
        assert self.lm_head is not None
        return self.lm_head.weight

    def project_to_logits(self, hidden: Tensor) -> Tensor:
        if self.tie_embeddings:
            return ops.linear(hidden, self.embed.weight)
        assert self.lm_head is not None
        return self.lm_head(hidden)

    def hidden_states(self, tokens: Tensor) -> Tensor:
        """``final_norm(blocks(embed(tokens)))``.

        Blocks that can leave their last residual add to the next norm
        (``supports_deferred_residual``) pass ``(stream, delta)`` along, so every add of the
        residual stream runs inside the following norm kernel, the final norm's included.
        """
        stream, pending = self.embed(tokens), None
        for block in self.blocks:
            if getattr(block, "supports_deferred_residual", False):
                stream, pending = block(stream, pending=pending, defer_residual=True)
                continue
            if pending is not None:
                stream, pending = stream + pending, None
            out = block(stream)
            stream = out[0] if isinstance(out, tuple) else out
        return add_then_norm(self.final_norm, stream, pending)[1]

    def forward(
        self,
        tokens: Tensor,
        *args: Any,
        targets: Tensor | None = None,
        ignore_index: int = -100,
        **kwargs: Any,
    ) -> Tensor:
        """Logits ``[B, S, V]``; with ``targets``, the unreduced next-token CE ``[B, S]``.

        The loss form never materializes logits when the head is a plain linear
        map (fused linear + CE on CUDA). It goes through ``forward`` so wrappers
        that hook ``__call__`` (FSDP unshard / reshard) see it.
        """
        del args, kwargs
        h = self.hidden_states(tokens)
        if targets is None:
            return self.project_to_logits(h)
        plain = self.tie_embeddings or (type(self.lm_head) is Linear and self.lm_head.bias is None)  # type: ignore[union-attr]
        if plain and not _is_dtensor(self.output_weight):
            return ops.linear_cross_entropy(h, self.output_weight, targets, ignore_index=ignore_index)
        return ops.cross_entropy(self.project_to_logits(h), targets, ignore_index=ignore_index)

    def token_loss(self, tokens: Tensor, targets: Tensor, *, ignore_index: int = -100) -> Tensor:
        """Unreduced next-token cross-entropy ``[B, S]`` (fp32); see :meth:`forward`."""
        return self(tokens, targets=targets, ignore_index=ignore_index)


def _is_dtensor(t: Tensor) -> bool:
    from torch.distributed.tensor import DTensor

    return isinstance(t, DTensor)
