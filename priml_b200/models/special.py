"""Identity / Skip / Sequential / SoftCap / ResidualMix
(``priml/model/special.py``, ``priml/model/sequential.py``,
``priml/model/softcap.py:38-94``, ``priml/model/residual_mix.py:22-80``)."""

from __future__ import annotations

import math
from dataclasses import KW_ONLY, field
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable, copy_tree
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, HasDepth, propagate_attr
from priml_b200.models.linear import Linear

__all__ = ["Identity", "ResidualMix", "Sequential", "Skip", "SoftCap"]


class Identity(nn.Identity):
    class Config(Fig["Identity"], kw_only=False):
        channels_in: int = -1
        channels_out: int = -1

        def finalize(self):  # noqa: ANN201
            if self.channels_in == -1:
                self.channels_in = self.channels_out
            if self.channels_out == -1:
                self.channels_out = self.channels_in
            return super().finalize()

    def __init__(self, config: Config | None = None) -> None:
        del config
        super().__init__()

    def reset_parameters(self) -> None:
        pass

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        return input


class Skip(nn.Module):
    """``x + inner(x)``."""

    class Config(Fig["Skip"], kw_only=False):
        inner: Makeable[nn.Module] | None = None

    def __init__(self, config: Config) -> None:
        if config.inner is None:
            raise ValueError("Must specify `inner`.")
        super().__init__()
        self.inner = config.inner.make()

    def reset_parameters(self) -> None:
        if hasattr(self.inner, "reset_parameters"):
            self.inner.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        return x + self.inner(x, *args, **kwargs)


class Sequential(nn.Sequential):
    """Chain of made elements; ``channels_in`` flows from each element's
    ``channels_out`` to the next (``priml/model/sequential.py:16-104``)."""

    class Config(Fig["Sequential"], kw_only=False):
        elements: list[Any] = field(default_factory=list)
        _: KW_ONLY
        channels_in: int = -1
        repeat: int = 1
        """Copies of ``elements`` to chain; with more than one, copy ``i`` gets ``depth = i``."""

        @property
        def channels_out(self) -> int:
            for e in reversed(self.elements):
                c = getattr(e, "channels_out", -1)
                if c != -1:
                    return c
            return self.channels_in

        def finalize(self):  # noqa: ANN201
            if self.repeat < 1:
                raise ValueError(f"repeat must be >= 1; got {self.repeat}.")
            if self.repeat > 1:
                base = self.elements if isinstance(self.elements, list) else [self.elements]
                flat = []
                for i in range(self.repeat):
                    for e in base:
                        e = copy_tree(e)
                        if isinstance(e, HasDepth):
                            e.depth = i
                        flat.append(e)
                self.elements = flat
                self.repeat = 1
            c = self.channels_in
            for e in self.elements:
                if c != -1:
                    propagate_attr(e, "channels_in", c, protocol=ChannelsIn)
                c = getattr(e, "channels_out", c)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__(*[e.make() for e in config.elements])

    def reset_parameters(self) -> None:
        for m in self:
            if hasattr(m, "reset_parameters"):
                m.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # type: ignore[override]
        for m in self:
            x = m(x, *args, **kwargs)
        return x


class SoftCap(nn.Module):
    """``cap * tanh(inner(x) / cap)`` evaluated in ``dtype`` (fp32 default)."""

    class Config(Fig["SoftCap"], kw_only=False):
        cap: float = 15.0
        _: KW_ONLY
        inner: Makeable[nn.Module] = field(default_factory=Linear.Config)
        channels_in: int = -1
        channels_out: int = -1
        dtype: torch.dtype | None = torch.float32

        def finalize(self):  # noqa: ANN201
            propagate_attr(self.inner, "channels_in", self.channels_in, protocol=ChannelsIn)
            propagate_attr(self.inner, "channels_out", self.channels_out, protocol=ChannelsOut)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if not math.isfinite(config.cap) or config.cap <= 0:
            raise ValueError(f"cap must be finite and positive; got {config.cap}.")
        self.cap = config.cap
        self.dtype = config.dtype
        self.inner = config.inner.make()

    @property
    def weight(self) -> Tensor:
        return self.inner.weight

    def reset_parameters(self) -> None:
        self.inner.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        out = self.inner(x)
        if self.dtype is not None:
            out = out.to(self.dtype)
        return self.cap * torch.tanh(out / self.cap)


class ResidualMix(nn.Module):
    """Per-layer ``running[i] * x + original[i] * x0``."""

    class Config(Fig["ResidualMix"], kw_only=False):
        num_layers: int = -1
        running: float = 1.0
        original: float = 0.1

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.num_layers <= 0:
            raise ValueError(f"num_layers must be positive; got {config.num_layers}.")
        self.config = config
        self.running = nn.Parameter(torch.empty(config.num_layers))
        self.original = nn.Parameter(torch.empty(config.num_layers))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        with torch.no_grad():
            self.running.fill_(self.config.running)
            self.original.fill_(self.config.original)

    def forward(self, x: Tensor, original: Tensor, *, layer: int) -> Tensor:
        return self.running[layer] * x + self.original[layer] * original
