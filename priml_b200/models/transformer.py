"""Residual transformer block: attention then feed-forward, each behind a norm.

Counterpart of ``priml/model/transformer.py:29-178``. The config fields and the
submodule names (``attn``, ``ffn``, ``norm1``, ``norm2``) are the reference's, so
configs and state dicts carry over; the forward pass is organised around the
residual stream instead.

Every residual add is done by the norm that reads its result. A pre-norm block
computes

    h  = x + pending          (fused into norm1)     n1 = norm1(h)
    h' = h + attn(n1)         (fused into norm2)     n2 = norm2(h')
    out = h' + ffn(n2)

and, when its caller asks (``defer_residual=True``), returns ``(h', ffn(n2))``
without adding them, so the next block's ``norm1`` (or the model's final norm)
performs that add too. On CUDA each fused add+norm is one kernel whose backward
also merges the residual-stream gradient with the norm's, so a block issues no
elementwise add or gradient-accumulation kernel of its own. Norms that cannot
fuse (another norm type, CPU tensors) get a plain add first: same values.
"""

from __future__ import annotations

from dataclasses import KW_ONLY, field
from typing import Any

import torch
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint as recompute

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

__all__ = ["TransformerBlock", "add_then_norm"]


def add_then_norm(norm: nn.Module, stream: Tensor, delta: Tensor | None) -> tuple[Tensor, Tensor]:
    """``(stream + delta, norm(stream + delta))``; one fused kernel when ``norm`` supports it."""
    fused = getattr(norm, "add_forward", None)
    if fused is not None:
        return fused(stream, delta)
    total = stream if delta is None else stream + delta
    return total, norm(total)


class TransformerBlock(nn.Module):
    """Pre-norm (default) or post-norm residual block; see the module docstring for the data flow."""

    supports_deferred_residual = True

    class Config(Fig["TransformerBlock"], kw_only=False):
        channels_in: int = -1
        """Residual-stream width."""
        _: KW_ONLY
        attn: Makeable[nn.Module] = field(default_factory=SelfAttention.Config)
        """Token-mixing sublayer."""
        ffn: Makeable[nn.Module] = field(default_factory=SwiGLU.Config)
        """Channel-mixing sublayer."""
        norm1: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        """Norm in front of (pre-norm) or behind (post-norm) ``attn``."""
        norm2: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        """Norm in front of or behind ``ffn``."""
        prenorm: bool = True
        """Normalize sublayer inputs (True) or residual sums (False)."""
        checkpoint: bool = False
        """Recompute the block in backward instead of keeping its activations."""
        depth: int = -1
        """Position in the stack, for depth-scaled initialisation (-1: none)."""

        @property
        def channels_out(self) -> int:
            return self.channels_in  # a residual block cannot change the stream's width

        @property
        def heads(self) -> int:
            return self.attn.heads if isinstance(self.attn, HeadGeometry) else 1

        @property
        def channels_head(self) -> int:
            return self.attn.channels_head if isinstance(self.attn, HeadGeometry) else self.channels_in

        def finalize(self):  # noqa: ANN201
            width, depth = self.channels_in, self.depth
            for sub in (self.attn, self.ffn, self.norm1, self.norm2):
                propagate_attr(sub, "channels_in", width, protocol=ChannelsIn)
                propagate_attr(sub, "channels_out", width, protocol=ChannelsOut)
                propagate_attr(sub, "depth", depth, protocol=HasDepth)
            if isinstance(self.ffn, ShardableConfig):
                self.ffn.shard = "colwise"  # tensor parallelism splits the FFN's hidden width
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
        for sub in self.children():
            reset = getattr(sub, "reset_parameters", None)
            if reset is not None:
                reset()

    # ------------------------------------------------------------------ forward
    def forward(
        self,
        x: Tensor,
        *args: Any,
        pending: Tensor | None = None,
        defer_residual: bool = False,
        **kwargs: Any,
    ) -> Any:
        """Residual stream in, residual stream out.

        ``pending`` is a residual delta the previous block left un-added (the stream is
        ``x + pending``). With ``defer_residual`` the result is ``(stream, delta)`` for the
        next block instead of their sum. When a ``cache`` keyword is given the attention's
        cache is returned beside the output, as in the reference.
        """
        if self.checkpoint and torch.is_grad_enabled():
            stream, delta, cache = recompute(self._mix, x, pending, args, kwargs, use_reentrant=False)
        else:
            stream, delta, cache = self._mix(x, pending, args, kwargs)
        if defer_residual:
            out: Any = (stream, delta)
        else:
            out = stream if delta is None else stream + delta
        if "cache" in kwargs and cache is not None:
            return out, cache
        return out

    def _mix(self, x: Tensor, pending: Tensor | None, args: tuple, kwargs: dict) -> tuple[Tensor, Tensor | None, Any]:
        if self.prenorm:
            stream, normed = add_then_norm(self.norm1, x, pending)
            mixed, cache = _split_cache(self.attn(normed, *args, **kwargs))
            stream, normed = add_then_norm(self.norm2, stream, mixed)
            return stream, self.ffn(normed), cache
        # post-norm: the norms' outputs are the stream, so nothing is left pending
        stream = x if pending is None else x + pending
        mixed, cache = _split_cache(self.attn(stream, *args, **kwargs))
        _, stream = add_then_norm(self.norm1, stream, mixed)
        _, stream = add_then_norm(self.norm2, stream, self.ffn(stream))
        return stream, None, cache


def _split_cache(result: Any) -> tuple[Tensor, Any]:
    """Attention returns a tensor, or ``(tensor, cache)`` when it keeps a KV cache."""
    if isinstance(result, Tensor):
        return result, None
    return result[0], result[1]
