"""Activation memoization strategies (``priml/train/activation.py:30-520``).

* ``DefaultActivationStorage`` keep everything (no-op).
* ``LayerActivationCheckpointing`` recompute every N-th block in backward.
* ``SelectiveActivationCheckpointing`` recompute a fraction of blocks of given types.
* ``QuantizedActivationStorage`` (alias ``Float8ActivationStorage``) store saved
  activations as e4m3 + per-tensor scale via ``saved_tensors_hooks``.
* ``QuantizedModuleActivationStorage`` quantize only the saved inputs of chosen
  module types (``nn.Conv2d``, ``nn.Linear``) through a per-module autograd function.
"""

from __future__ import annotations

from dataclasses import field
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint

from priml_b200.config import Fig

__all__ = [
    "DefaultActivationStorage",
    "Float8ActivationStorage",
    "LayerActivationCheckpointing",
    "QuantizedActivationStorage",
    "QuantizedModuleActivationStorage",
    "SelectiveActivationCheckpointing",
]


class DefaultActivationStorage:
    class Config(Fig["DefaultActivationStorage"]):
        pass

    def __init__(self, config: Any = None) -> None:
        del config

    def __call__(self, model: nn.Module) -> nn.Module:
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


def _quantize(t: Tensor, dtype_storage: torch.dtype) -> tuple[Tensor, Tensor]:
    """Per-tensor scaled cast: ``t ~= q * scale`` with ``|q| <= finfo(dtype_storage).max``.

    An all-zero tensor gets scale 1 (not 0/0), and its zeros come back exactly.
    """
    amax = t.detach().abs().amax().float()
    scale = amax / torch.finfo(dtype_storage).max
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    return (t.detach().float() / scale).to(dtype_storage), scale


class QuantizedActivationStorage:
    """Every saved activation of at least ``min_size`` elements held in a narrow float with a per-tensor scale.

    ``priml/train/activation.py:207-304``: the model's forward runs under
    ``saved_tensors_hooks`` that quantize on save and scale back on use, in
    ``dtype_compute`` when set, else the tensor's own dtype.
    """

    class Config(Fig["QuantizedActivationStorage"]):
        dtype_storage: torch.dtype = torch.float8_e4m3fn
        """Storage dtype of the saved activations."""
        dtype_compute: torch.dtype | None = None
        """Dtype the backward sees; None keeps each tensor's original dtype."""
        min_size: int = 4096
        """Tensors with fewer elements are saved as they are."""

    def __init__(self, config: Config | None = None) -> None:
        config = config or QuantizedActivationStorage.Config()
        self.dtype_storage = config.dtype_storage
        self.dtype_compute = config.dtype_compute
        self.min_size = config.min_size

    def _pack(self, t: Tensor) -> Any:
        if not t.is_floating_point() or t.numel() < self.min_size or t.dtype == self.dtype_storage:
            return t
        q, scale = _quantize(t, self.dtype_storage)
        return _Packed(q, scale, t.dtype, t.requires_grad)

    def _unpack(self, packed: Any) -> Tensor:
        if not isinstance(packed, _Packed):
            return packed
        out = packed.q.to(self.dtype_compute or packed.dtype) * packed.scale.to(self.dtype_compute or packed.dtype)
        return out.requires_grad_(packed.requires_grad)

    def __call__(self, model: nn.Module) -> nn.Module:
        orig = model.forward
        hooks = self

        def forward(*args: Any, **kwargs: Any) -> Any:
            with torch.autograd.graph.saved_tensors_hooks(hooks._pack, hooks._unpack):
                return orig(*args, **kwargs)

        model.forward = forward  # type: ignore[method-assign]
        return model


class _Packed:
    __slots__ = ("q", "scale", "dtype", "requires_grad")

    def __init__(self, q: Tensor, scale: Tensor, dtype: torch.dtype, requires_grad: bool) -> None:
        self.q, self.scale, self.dtype, self.requires_grad = q, scale, dtype, requires_grad


Float8ActivationStorage = QuantizedActivationStorage
"""The e4m3 default of :class:`QuantizedActivationStorage` (earlier name)."""


class _QuantizedInputOp(torch.autograd.Function):
    """``op(x, weight, bias)`` whose backward rebuilds ``x`` from a scaled narrow-float copy.

    ``op`` is ``"conv2d"`` (with stride / padding / dilation / groups) or ``"linear"``.
    """

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, bias: Tensor | None, op: str, conv: tuple,  # type: ignore[override]
                dtype_storage: torch.dtype, min_size: int) -> Tensor:  # fmt: skip
        out = F.conv2d(x, weight, bias, *conv) if op == "conv2d" else F.linear(x, weight, bias)
        if x.numel() >= min_size and x.is_floating_point():
            q, scale = _quantize(x, dtype_storage)
            ctx.save_for_backward(q, scale, weight)
            ctx.quantized = True
        else:
            ctx.save_for_backward(x, weight)
            ctx.quantized = False
        ctx.op, ctx.conv, ctx.x_dtype, ctx.x_shape, ctx.has_bias = op, conv, x.dtype, x.shape, bias is not None
        return out

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        if ctx.quantized:
            q, scale, weight = ctx.saved_tensors
            x = q.to(ctx.x_dtype) * scale.to(ctx.x_dtype)
        else:
            x, weight = ctx.saved_tensors
        dx = dw = db = None
        if ctx.op == "conv2d":
            stride, padding, dilation, groups = ctx.conv
            if ctx.needs_input_grad[0]:
                dx = torch.nn.grad.conv2d_input(ctx.x_shape, weight, g, stride, padding, dilation, groups)
            if ctx.needs_input_grad[1]:
                dw = torch.nn.grad.conv2d_weight(x, weight.shape, g, stride, padding, dilation, groups)
            if ctx.has_bias and ctx.needs_input_grad[2]:
                db = g.sum((0, 2, 3))
        else:
            g2 = g.reshape(-1, g.shape[-1])
            if ctx.needs_input_grad[0]:
                dx = (g2 @ weight.to(g.dtype)).view(ctx.x_shape)
            if ctx.needs_input_grad[1]:
                dw = (g2.T @ x.reshape(-1, x.shape[-1]).to(g.dtype)).to(weight.dtype)
            if ctx.has_bias and ctx.needs_input_grad[2]:
                db = g2.sum(0)
        return dx, dw, db, None, None, None, None


class QuantizedModuleActivationStorage:
    """Quantize only the inputs that chosen module types save for their backward.

    ``priml/train/activation.py:307-520`` wraps ``nn.Conv2d``. A per-module
    autograd function saves the input as a scaled narrow float and rebuilds it
    for the weight gradient, so nothing else in the graph pays for hooks.
    ``nn.Linear`` is supported too.
    """

    SUPPORTED: tuple[type[nn.Module], ...] = (nn.Conv2d, nn.Linear)

    class Config(Fig["QuantizedModuleActivationStorage"]):
        module_types: tuple[type[nn.Module], ...] = ()
        """Module classes whose saved inputs are quantized, e.g. ``(nn.Conv2d,)``."""
        dtype_storage: torch.dtype = torch.float8_e4m3fn
        """Storage dtype of the saved inputs."""
        min_size: int = 4096
        """Inputs with fewer elements are saved as they are."""

    def __init__(self, config: Config) -> None:
        if not config.module_types:
            raise ValueError("QuantizedModuleActivationStorage needs module_types, e.g. (nn.Conv2d,).")
        for t in config.module_types:
            if t not in self.SUPPORTED:
                raise ValueError(f"{t.__name__} is not supported; supported: {[c.__name__ for c in self.SUPPORTED]}.")
        self.module_types = tuple(config.module_types)
        self.dtype_storage = config.dtype_storage
        self.min_size = config.min_size

    def __call__(self, model: nn.Module) -> nn.Module:
        for module in model.modules():
            if type(module) in self.module_types:
                self._wrap(module)
        return model

    def _wrap(self, module: nn.Module) -> None:
        storage, min_size = self.dtype_storage, self.min_size
        if isinstance(module, nn.Conv2d):
            if module.padding_mode != "zeros":
                raise ValueError("only zero-padded Conv2d is supported")

            def conv_forward(x: Tensor, m: nn.Conv2d = module) -> Tensor:
                conv = (m.stride, m.padding, m.dilation, m.groups)
                return _QuantizedInputOp.apply(x, m.weight, m.bias, "conv2d", conv, storage, min_size)

            module.forward = conv_forward  # type: ignore[method-assign]
        else:

            def linear_forward(x: Tensor, m: nn.Linear = module) -> Tensor:  # type: ignore[assignment]
                return _QuantizedInputOp.apply(x, m.weight, m.bias, "linear", (), storage, min_size)

            module.forward = linear_forward  # type: ignore[method-assign]
