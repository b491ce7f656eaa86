"""Protocols shared by model blocks and the ``propagate_attr`` helper.

Mirrors the duck-typed contracts of the reference (``priml/model/custom_types.py:30-232``):
``ShardStyle``, the channel/depth/head-geometry protocols that parents use to push
shared dimensions into child configs, and ``propagate_attr`` itself.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any, Literal, Protocol, runtime_checkable

from torch import Tensor

__all__ = [
    "AttentionKernel",
    "ChannelsIn",
    "ChannelsInOut",
    "ChannelsOut",
    "HasDepth",
    "HeadGeometry",
    "RotaryFactors",
    "ShardStyle",
    "ShardableConfig",
    "TensorFn",
    "TensorModule",
    "propagate_attr",
]

ShardStyle = Literal["colwise", "rowwise", "vocab"]
"""Tensor-parallel shard style declared on a building-block config."""

TensorFn = Callable[[Tensor], Tensor]


class TensorModule(Protocol):
    """A module mapping a Tensor to a Tensor."""

    def __call__(self, x: Tensor, /, *args: Any, **kwargs: Any) -> Tensor: ...


@runtime_checkable
class RotaryFactors(Protocol):
    """Maps positions to the ``(cos, sin)`` half-dim factors of a rotation."""

    def __call__(self, positions: Tensor) -> tuple[Tensor, Tensor]: ...


@runtime_checkable
class AttentionKernel(Protocol):
    """``[..., S, H, D]`` q/k/v -> ``[..., S, H, D]`` attention output."""

    def __call__(self, q: Tensor, k: Tensor, v: Tensor, **kwargs: Any) -> Tensor: ...


@runtime_checkable
class HeadGeometry(Protocol):
    heads: int
    channels_head: int


@runtime_checkable
class HasDepth(Protocol):
    """Carries the layer index used for depth-scaled init."""

    depth: int


@runtime_checkable
class ChannelsIn(Protocol):
    channels_in: int


@runtime_checkable
class ChannelsOut(Protocol):
    channels_out: int


@runtime_checkable
class ChannelsInOut(ChannelsIn, ChannelsOut, Protocol):
    pass


@runtime_checkable
class ShardableConfig(Protocol):
    shard: ShardStyle | None


def propagate_attr(config: object, name: str, value: object, *, protocol: type | None = None) -> None:
    """Push ``value`` into ``config.name`` during a parent's ``finalize``.

    A child that does not satisfy ``protocol`` opts out silently. A child that
    satisfies it but cannot take the value raises ``AttributeError``. Read-only
    properties (a derived width such as ``channels_out == channels_in``) are left
    alone. Same contract as ``priml/model/custom_types.py:188-232``.
    """
    if config is None:
        return
    if protocol is not None and not isinstance(config, protocol):
        return
    if not hasattr(config, name):
        if protocol is None:
            return
        raise AttributeError(
            f"{type(config).__name__} satisfies {protocol.__name__} but has no attribute {name!r}"
        )
    descriptor = getattr(type(config), name, None)
    if isinstance(descriptor, property) and descriptor.fset is None:
        return
    setattr(config, name, value)
