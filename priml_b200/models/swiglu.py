"""Gated feed-forward (``priml/model/swiglu.py:32-278``).

``up_proj.weight`` is ``[2*hidden, C]`` with the GATE rows first, then the up
rows; ``out = down_proj(silu(gate) * up)``. On CUDA the gate/up product is a
fused kernel over the GEMM output (one read of ``[.., 2H]``, one write of
``[.., H]``); its backward recomputes ``silu`` from the saved pre-activation.
"""

from __future__ import annotations

from dataclasses import KW_ONLY
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig, Makeable, Makes
from priml_b200.math.basic import ceil_multiple
from priml_b200.models.custom_types import ChannelsIn, ShardStyle, TensorFn
from priml_b200.models.init import InitFn, kaiming_uniform, zeros
from priml_b200.models.linear import Linear

__all__ = ["SwiGLU", "SwiGLUReluSquared"]


class SwiGLU(nn.Module):
    class Config(Fig["SwiGLU"], kw_only=False):
        channels_in: int = -1
        channels_out: int = -1
        _: KW_ONLY
        channels_hidden: int = -1
        expansion: float = 8 / 3
        round_to: int = 256
        gate: bool = True
        bias: bool = False
        split_gate_projection: bool = False
        norm: Makeable[nn.Module] | None = None
        """Optional norm inside the gate branch (``sigmoid(g) * norm(g * x)``)."""
        act: TensorFn = nn.functional.silu
        depth: int = -1
        init_weight: InitFn = kaiming_uniform
        init_weight_out: InitFn | None = None
        shard: ShardStyle | None = None

        def finalize(self):  # noqa: ANN201
            if self.channels_in == -1:
                self.channels_in = self.channels_out
            if self.channels_out == -1:
                self.channels_out = self.channels_in
            if self.channels_hidden == -1:
                self.channels_hidden = int(ceil_multiple(self.channels_in * self.expansion, self.round_to))
            if isinstance(self.norm, ChannelsIn) and self.norm.channels_in == -1:
                self.norm.channels_in = self.channels_hidden
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        h = config.channels_hidden
        self.gate = config.gate
        self.depth = config.depth
        self.channels_hidden = h
        self.split_gate_projection = config.split_gate_projection
        self.shard = config.shard
        self.up_proj = Linear.Config(
            channels_in=config.channels_in,
            channels_out=2 * h if config.gate else h,
            bias=config.bias,
            depth=config.depth,
            init_weight=config.init_weight,
        ).make()
        self.down_proj = Linear.Config(
            channels_in=h,
            channels_out=config.channels_out,
            bias=config.bias,
            depth=config.depth,
            init_weight=config.init_weight_out or config.init_weight,
        ).make()
        self.act = config.act
        if config.norm is None:
            self.norm = None
        elif not self.gate:
            raise ValueError("Norm can only be specified when gate is enabled.")
        elif self.act is not nn.functional.silu:
            raise ValueError("Norm can only be specified when act is silu.")
        else:
            self.norm = config.norm.make()

    def reset_parameters(self) -> None:
        self.up_proj.reset_parameters()
        self.down_proj.reset_parameters()
        if self.norm is not None and hasattr(self.norm, "reset_parameters"):
            self.norm.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        if not self.gate:
            return self.down_proj(self.act(self.up_proj(x)))
        if self.split_gate_projection:
            gate, up = self._split_gate_projection(x)
        else:
            w = self.up_proj.weight
            fusable = self.norm is None and self.act is nn.functional.silu and self.up_proj.bias is None
            if fusable and type(self.up_proj) is Linear and not isinstance(w, _DTensorType()) and ops.use_native(x):
                down = self.down_proj
                wd = getattr(down, "weight", None)
                if type(down) is Linear and getattr(down, "bias", None) is None and not isinstance(wd, _DTensorType()):
                    return ops.swiglu_mlp(x, w, wd)
                return self.down_proj(ops.linear_swiglu(x, w))
            gate, up = self.up_proj(x).chunk(2, dim=-1)
        if self.norm is None:
            h = self.act(gate) * up
        else:
            h = torch.sigmoid(gate) * self.norm(gate * up)
        return self.down_proj(h)

    def tensor_parallel_style(self) -> Any:
        if self.split_gate_projection:
            raise NotImplementedError("SwiGLU tensor parallelism does not support split_gate_projection.")
        if self.norm is not None:
            raise NotImplementedError("SwiGLU tensor parallelism does not support a gate norm.")
        from priml_b200.parallel.tensor_parallel import SwiGLUParallel

        return SwiGLUParallel()

    def _split_gate_projection(self, x: Tensor) -> tuple[Tensor, Tensor]:
        c = self.channels_hidden
        w = self.up_proj.weight.to(x.dtype)
        b = None if self.up_proj.bias is None else self.up_proj.bias.to(x.dtype)
        gate = torch.matmul(x, w[:c].T)
        up = torch.matmul(x, w[c:].T)
        if b is not None:
            gate, up = gate + b[:c], up + b[c:]
        return gate, up


def _DTensorType() -> type:  # noqa: N802
    from torch.distributed.tensor import DTensor

    return DTensor


def _relu_squared(x: Tensor) -> Tensor:
    return torch.relu(x).square()


class SwiGLUReluSquared(SwiGLU):
    """Ungated ``down(relu(up(x))**2)`` with a zero-initialized output projection
    (``priml/model/swiglu.py:216-254``)."""

    class Config(Makes["SwiGLUReluSquared"], SwiGLU.Config, kw_only=False):
        gate: bool = False
        act: TensorFn = _relu_squared
        expansion: float = 4.0
        round_to: int = 1
        """No rounding: the hidden width is exactly ``expansion * channels_in``."""
        init_weight_out: InitFn | None = zeros
