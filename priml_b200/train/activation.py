"""Activation memoization strategies (``priml/train/activation.py:30-520``).

* ``DefaultActivationStorage`` keep everything (no-op).
* ``LayerActivationCheckpointing`` recompute every N-th block in backward.
* ``SelectiveActivationCheckpointing`` recompute a fraction of blocks of given types.
* ``Float8ActivationStorage`` store saved activations as e4m3 + per-tensor scale
  via ``saved_tensors_hooks`` (cast back on unpack).
"""

from __future__ import annotations

import contextlib
from dataclasses import field
from typing import Any

import torch
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint

from priml_b200.config import Fig

__all__ = [
    "DefaultActivationStorage",
    "Float8ActivationStorage",
    "LayerActivationCheckpointing",
    "SelectiveActivationCheckpointing",
]


class DefaultActivationStorage:
    class Config(Fig["DefaultActivationStorage"]):
        pass

    def __init__(self, config: Any = None) -> None:
        del config

    def __call__(self, model: nn.Module) -> nn.Module:
        return model


class _Checkpointed(nn.Module):
    def __init__(self, inner: nn.Module) -> None:
        super().__init__()
        self.inner = inner

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        if torch.is_grad_enabled():
            return checkpoint(self.inner, *args, use_reentrant=False, **kwargs)
        return self.inner(*args, **kwargs)


def _wrap_blocks(model: nn.Module, pick: Any) -> nn.Module:
    for name, mod in list(model.named_modules()):
        for child_name, child in list(mod.named_children()):
            if pick(child) and not isinstance(child, _Checkpointed):
                # Keep the state-dict keys: the wrapper forwards to the block in place.
                child.forward = _Checkpointed(child).forward.__get__(child)  # type: ignore[method-assign]
                _patch(child)
    return model


def _patch(block: nn.Module) -> None:
    orig = type(block).forward

    def forward(*args: Any, **kwargs: Any) -> Any:
        if torch.is_grad_enabled():
            return checkpoint(orig, block, *args, use_reentrant=False, **kwargs)
        return orig(block, *args, **kwargs)

    block.forward = forward  # type: ignore[method-assign]


class LayerActivationCheckpointing:
    class Config(Fig["LayerActivationCheckpointing"]):
        every: int = 1
        block_types: list[str] = field(default_factory=lambda: ["TransformerBlock"])

    def __init__(self, config: Config) -> None:
        self.config = config

    def __call__(self, model: nn.Module) -> nn.Module:
        blocks = [m for m in model.modules() if type(m).__name__ in self.config.block_types]
        for i, b in enumerate(blocks):
            if i % self.config.every == 0:
                _patch(b)
        return model


class SelectiveActivationCheckpointing:
    class Config(Fig["SelectiveActivationCheckpointing"]):
        fraction: float = 0.5
        block_types: list[str] = field(default_factory=lambda: ["TransformerBlock"])

    def __init__(self, config: Config) -> None:
        self.config = config

    def __call__(self, model: nn.Module) -> nn.Module:
        blocks = [m for m in model.modules() if type(m).__name__ in self.config.block_types]
        n = round(len(blocks) * self.config.fraction)
        for b in blocks[:n]:
            _patch(b)
        return model


class Float8ActivationStorage:
    """Saved activations held as float8_e4m3fn with a per-tensor amax scale."""

    class Config(Fig["Float8ActivationStorage"]):
        min_numel: int = 4096

    def __init__(self, config: Config | None = None) -> None:
        self.min_numel = (config or Float8ActivationStorage.Config()).min_numel

    def _pack(self, t: Tensor) -> Any:
        if not t.is_floating_point() or t.numel() < self.min_numel or t.dtype == torch.float8_e4m3fn:
            return t
        amax = t.detach().abs().amax().float().clamp_min(1e-12)
        scale = 448.0 / amax
        return ("fp8", (t.detach().float() * scale).to(torch.float8_e4m3fn), scale, t.dtype)

    def _unpack(self, packed: Any) -> Tensor:
        if isinstance(packed, tuple) and packed and packed[0] == "fp8":
            _, q, scale, dtype = packed
            return (q.float() / scale).to(dtype)
        return packed

    def __call__(self, model: nn.Module) -> nn.Module:
        orig = model.forward
        hooks = self

        def forward(*args: Any, **kwargs: Any) -> Any:
            with torch.autograd.graph.saved_tensors_hooks(hooks._pack, hooks._unpack):
                return orig(*args, **kwargs)

        model.forward = forward  # type: ignore[method-assign]
        return model


_ = (contextlib, _wrap_blocks)
