"""Normalization layers (``priml/model/norm.py:36-471``).

``RMSNorm`` runs the fused sm_100a kernel on CUDA (one row per warp group,
fp32 statistics, optional weight) and ATen's ``rms_norm`` on CPU.
"""

from __future__ import annotations

from dataclasses import KW_ONLY
from typing import Any, Protocol

import torch
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig

__all__ = [
    "BatchNorm",
    "BatchNorm2d",
    "BatchRenorm",
    "CenteredRMSNorm",
    "GroupNorm",
    "GroupNorm2d",
    "LayerNorm",
    "RMSNorm",
]



class NormProtocol(Protocol):
    """A normalization layer: called on a tensor, returns one of the same shape."""

    def __call__(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor: ...  # noqa: A002


class NormConfigProtocol(Protocol):
    """The fields every norm config shares, so a container can push its width (and whether the
    norm has a learned scale) into a nested norm config of any type."""

    channels_in: int
    elementwise_affine: bool

    def make(self) -> Any: ...

class RMSNorm(nn.RMSNorm):
    """Root-mean-square norm; ``eps=None`` takes the input dtype's epsilon."""

    class Config(Fig["RMSNorm"], kw_only=False):
        channels_in: int = -1
        """Normalized (last) dimension."""
        _: KW_ONLY
        eps: float | None = 1e-6
        """Added to the mean square; ``None`` means ``finfo(dtype).eps``."""
        elementwise_affine: bool = False
        """Learn a per-channel scale."""
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None

    def __init__(self, config: Config) -> None:
        super().__init__(
            normalized_shape=config.channels_in,
            eps=config.eps,
            elementwise_affine=config.elementwise_affine,
            device=config.device,
            dtype=config.dtype,
        )

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        return ops.rms_norm(input, self.weight, self.eps)

    def add_forward(self, x: Tensor, delta: Tensor | None) -> tuple[Tensor, Tensor]:
        """``(x + delta, norm(x + delta))`` with the add done inside the norm kernel on CUDA."""
        return ops.add_rms_norm(x, delta, self.weight, self.eps)


class CenteredRMSNorm(nn.Module):
    """RMSNorm scaled by ``1 + weight`` (weight starts at zero), computed in fp32."""

    class Config(Fig["CenteredRMSNorm"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        eps: float = 1e-6

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.eps = config.eps
        self.weight = nn.Parameter(torch.zeros(config.channels_in))

    def reset_parameters(self) -> None:
        nn.init.zeros_(self.weight)

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        # The gain is the zero-initialised offset plus one; the norm kernel accumulates in fp32
        # (on the host path the input is widened first), and the result keeps the input's dtype.
        gain = self.weight.float() + 1.0
        x = input if input.is_cuda else input.float()
        return ops.rms_norm(x, gain, self.eps).to(input.dtype)


class LayerNorm(nn.LayerNorm):
    class Config(Fig["LayerNorm"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        eps: float = 1e-5
        elementwise_affine: bool = False
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None

    def __init__(self, config: Config) -> None:
        super().__init__(
            normalized_shape=config.channels_in,
            eps=config.eps,
            elementwise_affine=config.elementwise_affine,
            device=config.device,
            dtype=config.dtype,
        )

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        return super().forward(input)


class BatchNorm(nn.BatchNorm1d):
    """Batch norm over every axis but the last (features-last input)."""

    class Config(Fig["BatchNorm"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        momentum: float = 0.1
        eps: float = 1e-5
        elementwise_affine: bool = False
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None

    def __init__(self, config: Config) -> None:
        super().__init__(
            config.channels_in,
            momentum=config.momentum,
            eps=config.eps,
            affine=config.elementwise_affine,
            device=config.device,
            dtype=config.dtype,
        )

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        # BatchNorm1d takes (N, C) or (N, C, L): present the features-last input channels-first,
        # merging any extra middle axes into L, and turn the result back.
        x = input if input.dim() <= 3 else input.flatten(1, -2)
        return super().forward(x.movedim(-1, 1)).movedim(1, -1).reshape(input.shape)


class BatchRenorm(nn.Module):
    """Batch renormalization (Ioffe 2017, arXiv:1702.03275): batch statistics
    corrected toward the running ones by a clipped, detached affine term once
    ``warmup_steps`` updates have accumulated (``priml/model/norm.py:190-345``)."""

    class Config(Fig["BatchRenorm"]):
        channels_in: int = 1
        momentum: float = 0.999
        eps: float = 1e-3
        warmup_steps: int = 1_000
        max_ratio: float = 3.0
        max_drift: float = 5.0

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.channels_in <= 0:
            raise ValueError("channels_in must be positive")
        if config.max_ratio < 1.0:
            raise ValueError("max_ratio must be at least one")
        if config.max_drift < 0.0:
            raise ValueError("max_drift must be non-negative")
        if not 0.0 <= config.momentum < 1.0:
            raise ValueError("momentum must be in [0, 1)")
        self.config = config
        self.weight = nn.Parameter(torch.ones(config.channels_in))
        self.bias = nn.Parameter(torch.zeros(config.channels_in))
        self.register_buffer("running_mean", torch.zeros(config.channels_in))
        self.register_buffer("running_var", torch.ones(config.channels_in))
        self.register_buffer("steps", torch.zeros((), dtype=torch.int64))

    def forward(self, x: Tensor) -> Tensor:
        c = self.config
        if not self.training:
            return self._affine(x, self.running_mean, self.running_var)
        axes = tuple(range(x.dim() - 1))
        mean = x.mean(dim=axes)
        var = ((x - mean) ** 2).mean(dim=axes)
        use_mean, use_var = mean, var
        if bool(self.steps >= c.warmup_steps):
            dev = (var + c.eps).sqrt()
            run_dev = (self.running_var + c.eps).sqrt()
            r = (dev / run_dev).detach().clamp(1.0 / c.max_ratio, c.max_ratio)
            d = ((mean - self.running_mean) / run_dev).detach().clamp(-c.max_drift, c.max_drift)
            use_mean, use_var = mean - d * dev / r, var / r**2
        with torch.no_grad():
            self.running_mean.mul_(c.momentum).add_(mean, alpha=1.0 - c.momentum)
            self.running_var.mul_(c.momentum).add_(var, alpha=1.0 - c.momentum)
            self.steps.add_(1)
        return self._affine(x, use_mean, use_var)

    def _affine(self, x: Tensor, mean: Tensor, var: Tensor) -> Tensor:
        return (x - mean) / (var + self.config.eps).sqrt() * self.weight + self.bias


class BatchNorm2d(nn.BatchNorm2d):
    class Config(Fig["BatchNorm2d"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        momentum: float = 0.1
        eps: float = 1e-5
        elementwise_affine: bool = False
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None

    def __init__(self, config: Config) -> None:
        super().__init__(
            config.channels_in,
            momentum=config.momentum,
            eps=config.eps,
            affine=config.elementwise_affine,
            device=config.device,
            dtype=config.dtype,
        )

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        return super().forward(input)


class GroupNorm2d(nn.GroupNorm):
    """Channels-first group norm (no running statistics)."""

    class Config(Fig["GroupNorm2d"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        num_groups: int = 8
        eps: float = 1e-5
        elementwise_affine: bool = False
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None

    def __init__(self, config: Config) -> None:
        super().__init__(
            config.num_groups,
            config.channels_in,
            eps=config.eps,
            affine=config.elementwise_affine,
            device=config.device,
            dtype=config.dtype,
        )

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        return super().forward(input)


class GroupNorm(nn.GroupNorm):
    """Features-last group norm over ``[..., L, C]``."""

    class Config(Fig["GroupNorm"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        num_groups: int = 8
        eps: float = 1e-5
        elementwise_affine: bool = False
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None

    def __init__(self, config: Config) -> None:
        super().__init__(
            config.num_groups,
            config.channels_in,
            eps=config.eps,
            affine=config.elementwise_affine,
            device=config.device,
            dtype=config.dtype,
        )

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        shape = input.shape
        x = input.reshape(-1, *shape[-2:]).movedim(-2, -1)
        return super().forward(x).movedim(-2, -1).reshape(shape)
