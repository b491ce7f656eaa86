"""Grid-puzzle solver with an optional latent recurrence (``priml/baselines/sudoku/model.py:1-552``).

``SudokuNet`` embeds a grid (plus optional prefix tokens), runs a block stack
over it, and reads token logits from every position and a halt logit from
position 0. The stack is any ``(x, *args, **kwargs) -> x`` module (transformer
or MLP-mixer); blocks are POST-norm because a recurrence feeds the stack its
own output and pre-norm lets the carried residual stream grow without bound.

One *core* application refines two latents of shape ``[B, S, C]``::

    for _ in range(fast_cycles):
        z_fast = mix(z_fast + z_slow + input)
    z_slow = mix(z_slow + z_fast)

:class:`DeepRecurrence` runs ``slow_cycles`` cores, all but the last under
``no_grad``: backpropagation goes through ONE core whatever the depth, so
memory and backward time are flat in the cycle count. Without a recurrence the
core runs once with one fast cycle.

On CUDA every block runs on this framework's kernels (tcgen05 GEMMs, fused
RMSNorm, the flash-attention kernel for the bidirectional 81- or 900-token
attention); the no-grad cycles keep no activations, so a deep rollout costs
forward FLOPs only.
"""

from __future__ import annotations

import copy
import functools
import logging
from dataclasses import field
from typing import Any, NamedTuple, Protocol, runtime_checkable

import torch
from torch import Tensor, nn

from priml_b200.baselines.sudoku.embedding import GridEmbedding, HasHiddenSize
from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsIn
from priml_b200.models.init import truncated_normal
from priml_b200.models.linear import Linear
from priml_b200.models.special import Sequential
from priml_b200.models.transformer import TransformerBlock

__all__ = ["CoreOutput", "DeepRecurrence", "ForwardOutput", "SudokuNet", "corrected_fan_in_normal"]

logger = logging.getLogger(__name__)


def corrected_fan_in_normal(w: Tensor, *, depth: int = -1) -> None:
    """Truncated normal with realized std ``fan_in ** -0.5``."""
    del depth
    truncated_normal(w, std=w.shape[-1] ** -0.5, depth=-1, variance_correction=True)


class CoreOutput(NamedTuple):
    logits: Tensor
    """``[B, S, V]`` over the whole sequence (prefix included)."""
    halt: Tensor
    """``[B]`` fp32 halt logit read at position 0."""
    z_slow: Tensor
    z_fast: Tensor


class ForwardOutput(NamedTuple):
    logits: Tensor
    """``[B, grid_len, V]``, prefix positions stripped."""
    halt: Tensor
    z_slow: Tensor
    """``[B, S, C]``, detached for carrying."""
    z_fast: Tensor
    all_logits: tuple[Tensor, ...] = ()
    """Per-slow-cycle logits when asked for (``collect_intermediates``)."""


@runtime_checkable
class HasNumTokens(Protocol):
    num_tokens: int


@runtime_checkable
class HasParts(Protocol):
    parts: list[Any]


def _count_prefix_tokens(prefix: Any) -> int:
    if prefix is None:
        return 0
    if isinstance(prefix, HasParts):
        return sum(_count_prefix_tokens(p) for p in prefix.parts)
    if isinstance(prefix, HasNumTokens):
        return int(prefix.num_tokens)
    raise ValueError(
        f"{type(prefix).__name__} fills the prefix slot but declares no num_tokens; "
        "add the field or set num_prefix_tokens."
    )


class DeepRecurrence(nn.Module):
    """``slow_cycles`` core applications, the first ``slow_cycles - 1`` without gradient."""

    class Config(Fig["DeepRecurrence"]):
        slow_cycles: int = 6
        fast_cycles: int = 9

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.slow_cycles < 1 or config.fast_cycles < 1:
            raise ValueError(f"slow_cycles and fast_cycles must be >= 1; got {config.slow_cycles}, {config.fast_cycles}.")
        self.config = config

    def forward(self, core: Any, input_emb: Tensor, z_slow: Tensor, z_fast: Tensor, *,
                collect_intermediates: bool = False) -> ForwardOutput:  # fmt: skip
        kept: list[Tensor] = []
        with torch.no_grad():
            x = input_emb.detach()
            for _ in range(self.config.slow_cycles - 1):
                out = core(x, z_slow.detach(), z_fast.detach())
                z_slow, z_fast = out.z_slow, out.z_fast
                if collect_intermediates:
                    kept.append(out.logits)
        last = core(input_emb, z_slow, z_fast)
        if collect_intermediates:
            kept.append(last.logits.detach())
        return ForwardOutput(last.logits, last.halt, last.z_slow, last.z_fast, tuple(kept))


def _latent_init(c: int) -> Tensor:
    w = torch.empty(1, c)
    truncated_normal(w, std=1.0, depth=-1, variance_correction=True)
    return w


class SudokuNet(nn.Module):
    class Config(Fig["SudokuNet"]):
        hidden_size: int = 512
        num_layers: int = 2
        embedding: Makeable[GridEmbedding] = field(default_factory=GridEmbedding.Config)
        block: Makeable[nn.Module] = field(default_factory=lambda: TransformerBlock.Config(prenorm=False))
        recurrence: Makeable[DeepRecurrence] | None = None
        prefix: Makeable[nn.Module] | None = None
        num_prefix_tokens: int = -1
        """Prefix tokens; -1 counts them from the prefix config (0 without one)."""
        vocab_size: int = 11
        halt_outputs: int = 2
        """Halt-head width; only column 0 is read (two columns keep checkpoint shapes)."""
        halt_init_bias: float = -5.0

        @property
        def grid_len(self) -> int:
            return self.embedding.grid_len

        @property
        def total_seq_len(self) -> int:
            n = _count_prefix_tokens(self.prefix) if self.num_prefix_tokens == -1 else self.num_prefix_tokens
            return n + self.grid_len

        def finalize(self):  # noqa: ANN201
            emb = self.embedding
            if emb.hidden_size == -1:
                emb.hidden_size = self.hidden_size
            emb.vocab_size = self.vocab_size
            if isinstance(self.block, ChannelsIn) and self.block.channels_in == -1:
                self.block.channels_in = self.hidden_size
            if isinstance(self.prefix, HasHiddenSize) and self.prefix.hidden_size == -1:
                self.prefix.hidden_size = self.hidden_size
            if self.num_prefix_tokens == -1:
                self.num_prefix_tokens = _count_prefix_tokens(self.prefix)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.config = config
        c = config.hidden_size
        self.embedding = config.embedding.make()
        self.head = Linear.Config(c, config.vocab_size, bias=False, init_weight=corrected_fan_in_normal).make()
        self.halt_head = Linear.Config(
            c, config.halt_outputs, bias=True, init_weight=nn.init.zeros_,
            init_bias=functools.partial(nn.init.constant_, val=config.halt_init_bias),
        ).make()  # fmt: skip
        self.reasoning = Sequential.Config([copy.deepcopy(config.block)], channels_in=c, repeat=config.num_layers).make()
        self.prefix = config.prefix.make() if config.prefix is not None else None
        self.slow_init = nn.Buffer(_latent_init(c), persistent=True)
        self.fast_init = nn.Buffer(_latent_init(c), persistent=True)
        self.recurrence = config.recurrence.make() if config.recurrence is not None else None
        # an empty persistent buffer that the reference's checkpoints carry (``_dummy``): kept so that
        # its state dicts load strictly
        self._dummy = nn.Buffer(torch.empty(0), persistent=True)
        logger.info("sudoku model parameters: %.2fM", sum(p.numel() for p in self.parameters()) / 1e6)

    @property
    def device(self) -> torch.device:
        return self.slow_init.device

    @property
    def fast_cycles(self) -> int:
        return self.recurrence.config.fast_cycles if self.recurrence is not None else 1

    def init_latents(self, batch_size: int) -> tuple[Tensor, Tensor]:
        s = self.config.total_seq_len
        return (self.slow_init.expand(batch_size, s, -1).contiguous(),
                self.fast_init.expand(batch_size, s, -1).contiguous())  # fmt: skip

    def _mix(self, z: Tensor) -> Tensor:
        return self.reasoning(z, cos_sin=None)

    def core(self, input_emb: Tensor, z_slow: Tensor, z_fast: Tensor) -> CoreOutput:
        injected = z_slow + input_emb
        for _ in range(self.fast_cycles):
            z_fast = self._mix(z_fast + injected)
        z_slow = self._mix(z_slow + z_fast)
        logits = self.head(z_slow)
        halt = self.halt_head(z_slow[:, 0]).float()
        halt = halt.squeeze(-1) if self.config.halt_outputs == 1 else halt[..., 0]
        return CoreOutput(logits, halt, z_slow, z_fast)

    def embed(self, tokens: Tensor, prefix_kwargs: dict[str, Any]) -> Tensor:
        x = self.embedding(tokens)
        if self.prefix is None:
            return x
        p = self.prefix(tokens.shape[0], **prefix_kwargs)
        return torch.cat([p.to(x.dtype), x], dim=1)

    def forward(self, tokens: Tensor, z_slow: Tensor | None = None, z_fast: Tensor | None = None, *,
                collect_intermediates: bool = False, **prefix_kwargs: Any) -> ForwardOutput:  # fmt: skip
        x = self.embed(tokens, prefix_kwargs)
        if z_slow is None or z_fast is None:
            z_slow, z_fast = self.init_latents(tokens.shape[0])
        if self.recurrence is None:
            o = self.core(x, z_slow, z_fast)
            res = ForwardOutput(o.logits, o.halt, o.z_slow, o.z_fast,
                                (o.logits.detach(),) if collect_intermediates else ())  # fmt: skip
        else:
            res = self.recurrence(self.core, x, z_slow, z_fast, collect_intermediates=collect_intermediates)
        n = self.config.num_prefix_tokens
        logits, kept = res.logits, res.all_logits
        if n:
            logits, kept = logits[:, n:], tuple(t[:, n:] for t in kept)
        return ForwardOutput(logits, res.halt, res.z_slow.detach(), res.z_fast.detach(), kept)
