"""Linear layers (``priml/model/linear.py:24-199``).

``Linear`` keeps ``nn.Linear``'s parameter layout (``weight [out, in]``) so
checkpoints interchange; ``EnsembleLinear`` holds ``[E, out, in]`` (e.g. fused
per-head QKV). Both run through :func:`priml_b200.ops.linear`, i.e. the tcgen05
GEMM on CUDA.
"""

from __future__ import annotations

from dataclasses import KW_ONLY
from functools import partial
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig
from priml_b200.models.custom_types import ShardStyle
from priml_b200.models.init import InitFn, call_init, kaiming_uniform

__all__ = ["EnsembleLinear", "Linear"]


class Linear(nn.Linear):
    """``nn.Linear`` with injected init, depth scaling and a TP shard style."""

    class Config(Fig["Linear"], kw_only=False):
        channels_in: int = -1
        channels_out: int = -1
        _: KW_ONLY
        bias: bool = False
        depth: int = -1
        """Block index for depth-scaled init (-1 = none)."""
        device: torch.device | str | None = None
        dtype: torch.dtype | None = None
        init_weight: InitFn = kaiming_uniform
        init_bias: InitFn = nn.init.zeros_
        shard: ShardStyle | None = None
        """Tensor-parallel style over the ``tp`` mesh dim (None replicates)."""

        def finalize(self):  # noqa: ANN201
            if self.channels_in == -1:
                self.channels_in = self.channels_out
            if self.channels_out == -1:
                self.channels_out = self.channels_in
            return super().finalize()

    def __init__(self, config: Config) -> None:
        self.depth = config.depth
        self._init_weight = config.init_weight
        self._init_bias = config.init_bias
        self.shard = config.shard
        super().__init__(
            in_features=config.channels_in,
            out_features=config.channels_out,
            bias=config.bias,
            device=config.device,
            dtype=config.dtype,
        )

    def reset_parameters(self) -> None:
        if not hasattr(self, "_init_weight"):
            return super().reset_parameters()
        call_init(self._init_weight, self.weight, depth=self.depth)
        if self.bias is not None:
            call_init(self._init_bias, self.bias, depth=self.depth)
        return None

    def forward(self, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
        del args, kwargs
        return ops.linear(input, self.weight, self.bias)


class EnsembleLinear(nn.Module):
    """Linear with an ensemble axis: weight ``[E, out, in]``, output ``[..., E, out]``.

    Computed as one GEMM against ``weight.reshape(E*out, in)``.
    """

    class Config(Fig["EnsembleLinear"], kw_only=False):
        channels_in: int = -1
        channels_out: int = -1
        _: KW_ONLY
        num_ensemble: int = -1
        bias: bool = False
        depth: int = -1
        init_weight: InitFn = kaiming_uniform
        shard: ShardStyle | None = None

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.shard = config.shard
        self.weight = nn.Parameter(torch.empty(config.num_ensemble, config.channels_out, config.channels_in))
        self.bias: nn.Parameter | None = (
            nn.Parameter(torch.zeros(config.num_ensemble, config.channels_out)) if config.bias else None
        )
        self.depth = config.depth
        self._init_weight = config.init_weight
        self.reset_parameters()

    def reset_parameters(self) -> None:
        for i in range(self.weight.shape[0]):
            call_init(self._init_weight, self.weight.data[i], depth=self.depth)
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        w = self.weight
        out = ops.linear(x, w.reshape(-1, w.shape[-1]), None if self.bias is None else self.bias.reshape(-1))
        return out.reshape(*x.shape[:-1], *w.shape[:-1])

    def tensor_parallel_style(self) -> Any:
        """Shard the ensemble (head) axis; replicate the input."""
        from priml_b200.parallel.tensor_parallel import EnsembleParallel

        return EnsembleParallel()


_ = partial
