"""NanoChat decoder (``priml/baselines/nanochat/model.py:57-491``).

Embed, run every block over a residual stream re-mixed with the normalized
token embedding at each layer, and project to soft-capped vocabulary logits.
What the stack decides, because it depends on position in depth:

* which layers attend over a window and which over the whole context (the
  attention's ``S`` / ``L`` pattern; the last layer is always long);
* which layers read a value embedding: every ``value_embedding_stride``-th
  layer counted back from the last, so the rule survives a change of depth;
* the value-embedding tables, one per reading layer, as wide as the attention's
  values (``heads * channels_head``).

B200 path: the blocks run the tcgen05 GEMMs and flash attention (windowed);
:meth:`token_loss` computes the soft-capped cross-entropy straight from the
final hidden states with the fused linear + CE kernel, so the ``[B, S, V]``
fp32 logits the reference materializes are never written.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import field
from functools import partial
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, propagate_attr
from priml_b200.models.embedding import Embedding, NarrowEmbedding
from priml_b200.models.init import normal, unit_fan_in_uniform
from priml_b200.models.linear import Linear
from priml_b200.models.norm import RMSNorm
from priml_b200.models.rope import RoPE
from priml_b200.models.special import ResidualMix, SoftCap
from priml_b200.models.swiglu import SwiGLUReluSquared
from priml_b200.models.transformer import TransformerBlock
from priml_b200.models.value_gated_attention import ValueGatedAttention

__all__ = ["NanoChatLM"]


def _head_shape(block: Any, channels_in: int) -> tuple[int, int]:
    """``(channels_head, heads * channels_head)`` of a block's attention."""
    attn = getattr(block, "attn", None)
    heads, head = getattr(attn, "heads", -1), getattr(attn, "channels_head", -1)
    if heads is None or head is None or heads <= 0 or head <= 0:
        return channels_in, channels_in
    return head, heads * head


class NanoChatLM(nn.Module):
    """Decoder-only transformer with windowed attention and value embeddings."""

    class Config(Fig["NanoChatLM"]):
        vocab_size: int = 8192
        max_seq_len: int = 2048
        """Context length, and the long attention window."""
        channels_in: int = 512
        num_layers: int = 8
        block: Any = field(
            default_factory=lambda: TransformerBlock.Config(
                attn=ValueGatedAttention.Config(), ffn=SwiGLUReluSquared.Config()
            )
        )
        """Block template (copied ``num_layers`` times) or a per-layer list."""
        value_embedding_stride: int = 0
        """Every Nth layer, counted back from the last, reads a value embedding (0: none)."""
        embedding: Makeable[nn.Module] = field(
            default_factory=lambda: NarrowEmbedding.Config(inner=Embedding.Config(init_weight=partial(normal, std=1.0)))
        )
        norm: Makeable[nn.Module] = field(default_factory=lambda: RMSNorm.Config(eps=None))
        lm_head: Makeable[nn.Module] = field(
            default_factory=lambda: SoftCap.Config(inner=Linear.Config(bias=False, init_weight=partial(normal, std=0.001)))
        )
        rope: RoPE.Config = field(default_factory=lambda: RoPE.Config(hf_inv_freq=True))
        mix: ResidualMix.Config = field(default_factory=ResidualMix.Config)

        @property
        def template(self) -> Any:
            """The block config every layer copies when ``block`` is a single transformer block.

            A per-layer list (or a block that is not a transformer) has no single template, so
            asking for one is an error rather than a silent pick of the first layer.
            """
            from priml_b200.models.transformer import TransformerBlock

            if not isinstance(self.block, TransformerBlock.Config):
                raise TypeError(f"block is {type(self.block).__name__}, not one TransformerBlock.Config: no single template")
            return self.block

        @property
        def value_embedding_layers(self) -> list[int]:
            if self.value_embedding_stride <= 0:
                return []
            return sorted(range(self.num_layers - 1, -1, -self.value_embedding_stride))

        def finalize(self):  # noqa: ANN201
            if self.vocab_size <= 0:
                raise ValueError(f"vocab_size must be positive; got {self.vocab_size}.")
            if self.max_seq_len < 2:
                raise ValueError(f"max_seq_len must be at least two; got {self.max_seq_len}.")
            if self.num_layers <= 0 or self.channels_in <= 0:
                raise ValueError("num_layers and channels_in must be positive.")
            if self.value_embedding_stride < 0:
                raise ValueError(f"value_embedding_stride must be nonnegative; got {self.value_embedding_stride}.")
            if not isinstance(self.block, Sequence):
                self.block = [self.block.copy_tree() for _ in range(self.num_layers)]
            if len(self.block) != self.num_layers:
                raise ValueError(f"block names {len(self.block)} layers for num_layers={self.num_layers}.")
            gated = set(self.value_embedding_layers)
            last = self.num_layers - 1
            for layer, block in enumerate(self.block):
                propagate_attr(block, "channels_in", self.channels_in, protocol=ChannelsIn)
                propagate_attr(block, "channels_out", self.channels_in, protocol=ChannelsOut)
                propagate_attr(block, "depth", layer)
                attn = getattr(block, "attn", None)
                if isinstance(attn, ValueGatedAttention.Config):
                    attn.max_seq_len = self.max_seq_len
                    if layer == last:
                        attn.window = self.max_seq_len
                    attn.gated = layer in gated
            propagate_attr(self.embedding, "channels_out", self.channels_in)
            propagate_attr(self.embedding, "num_embeddings", self.vocab_size)
            propagate_attr(self.lm_head, "channels_in", self.channels_in)
            propagate_attr(self.lm_head, "channels_out", self.vocab_size)
            propagate_attr(self.norm, "channels_in", self.channels_in, protocol=ChannelsIn)
            self.mix.num_layers = self.num_layers
            heads = {getattr(getattr(b, "attn", None), "channels_head", self.channels_in) for b in self.block}
            if len(heads) > 1:
                raise ValueError(f"every block must use the same attention head width; got {sorted(heads)}.")
            self.rope.channels_head = next(iter(heads))  # the model builds the factors, the heads consume them
            out = super().finalize()
            # after the cascade, when every attention has derived its head count
            shapes = {_head_shape(b, out.channels_in) for b in out.block}
            if len(shapes) > 1:
                raise ValueError(
                    "every block must declare the same attention head geometry (the value embeddings and "
                    f"rotary factors are shared); got {sorted(shapes)}."
                )
            return out

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.config = config
        _, width = _head_shape(config.block[0], config.channels_in)
        # construction order fixes the global-RNG draw order: tokens, head, blocks, value embeddings
        self.embed = config.embedding.make()
        self.lm_head = config.lm_head.make()
        self.blocks = nn.ModuleList([b.make() for b in config.block])
        self.value_embeds = nn.ModuleDict({str(i): self._value_table(config, width) for i in config.value_embedding_layers})
        self.norm_embed = config.norm.make()
        self.norm_out = config.norm.make()
        self.mix = config.mix.make()
        self.rope = config.rope.make()
        self._rotation: tuple[Tensor, Tensor] | None = None

    @staticmethod
    def _value_table(config: Config, width: int) -> nn.Module:
        table = NarrowEmbedding.Config(inner=Embedding.Config(init_weight=unit_fan_in_uniform))
        table.channels_out = width
        table.num_embeddings = config.vocab_size
        if isinstance(config.embedding, NarrowEmbedding.Config):
            table.dtype = config.embedding.dtype
        return table.make()

    def reset_parameters(self) -> None:
        for m in (self.embed, self.lm_head, self.norm_embed, self.norm_out, self.mix, *self.blocks,
                  *self.value_embeds.values()):  # fmt: skip
            if hasattr(m, "reset_parameters"):
                m.reset_parameters()
        self._rotation = None

    def _rotation_table(self, length: int, device: torch.device) -> tuple[Tensor, Tensor]:
        """Rotation factors built once for ``max_seq_len`` on this device and sliced."""
        if self._rotation is None or self._rotation[0].device != device:
            self._rotation = self.rope(torch.arange(self.config.max_seq_len, device=device))
        cos, sin = self._rotation
        return cos[:length], sin[:length]

    def hidden(self, tokens: Tensor) -> Tensor:
        """Final normalized hidden states ``[B, S, C]`` (before the vocabulary projection)."""
        length = tokens.shape[-1]
        if length > self.config.max_seq_len:
            raise ValueError(f"Input length {length} exceeds max_seq_len={self.config.max_seq_len}.")
        cos_sin = self._rotation_table(length, tokens.device)
        x = self.norm_embed(self.embed(tokens))
        original = x
        for layer, block in enumerate(self.blocks):
            x = self.mix(x, original, layer=layer)
            name = str(layer)
            ve = self.value_embeds[name](tokens) if name in self.value_embeds else None
            x = block(x, cos_sin=cos_sin, value_embedding=ve)
        return self.norm_out(x)

    def forward(self, tokens: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        """``[B, S]`` token ids to ``[B, S, vocab]`` soft-capped logits (fp32)."""
        del args, kwargs
        return self.lm_head(self.hidden(tokens))

    def token_loss(self, tokens: Tensor, targets: Tensor, *, ignore_index: int = -1) -> Tensor:
        """Unreduced next-token cross-entropy ``[B, S]`` (fp32) without a logits tensor."""
        h = self.hidden(tokens)
        head = self.lm_head
        cap = head.cap if isinstance(head, SoftCap) else None
        weight = head.weight
        loss = ops.linear_cross_entropy(h.reshape(-1, h.shape[-1]), weight, targets.reshape(-1),
                                        ignore_index=ignore_index, softcap=cap)  # fmt: skip
        return loss.view(targets.shape)

    def flops_per_token(self) -> int:
        """Forward + backward FLOPs per token: 6 x matrix parameters + 12 x inner width x window per layer."""
        gathered = {id(p) for m in (self.embed, *self.value_embeds.values(), self.mix) for p in m.parameters()}
        matrix = sum(p.numel() for p in self.parameters() if id(p) not in gathered)
        _, inner = _head_shape(self.config.block[0], self.config.channels_in)
        attention = 0
        for b in self.blocks:
            window = getattr(getattr(getattr(b, "attn", None), "config", None), "window", None)
            if not isinstance(window, int):
                raise TypeError(f"{type(b).__name__} declares no attention window.")
            attention += 12 * inner * window
        return 6 * matrix + attention
