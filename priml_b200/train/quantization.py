"""Low-precision training of linear layers (``priml/train/quantization.py:22-149``).

``Float8ModelQuantization`` keeps the reference's config surface (``recipe``,
``module_filter``, ``enable_fsdp_float8_all_gather``) but is built on MXFP8
(OCP microscaling: E4M3 values with one E8M0 scale per 32 elements along each
GEMM's contraction dimension) run by the block-scaled tcgen05 kernels of
``ops/csrc/mxfp8.cu`` instead of torchao's tensorwise / rowwise scaling:

* ``mxfp8`` (default), ``tensorwise`` and ``rowwise``: forward, dgrad and wgrad
  in MXFP8. A 32-element block scale is finer than a row or tensor scale, so the
  two reference recipes map to the same, more accurate, block scaling.
* ``rowwise_gw_hp``: forward and dgrad in MXFP8, weight gradient in bf16, as the
  reference's recipe of that name keeps the weight gradient in high precision.

Conversion swaps each selected ``nn.Linear`` (default filter: bias-free, both
dimensions multiples of 32) to a subclass whose forward runs
:func:`priml_b200.ops.mx.mx_linear`; parameters and state-dict keys are
unchanged, so checkpoints move freely between quantized and bf16 models.
``enable_fsdp_float8_all_gather`` is accepted and has no effect: with resident
weights the fused sharded strategy all-gathers only the optimizer's bf16 output,
and with sharded weights (``shard_params``) its per-block bf16 gather runs on the
copy engines a block ahead, off the critical path, so fp8 bytes would not shorten
the step.
"""

from __future__ import annotations

import logging
from collections.abc import Callable
from typing import Any

from torch import Tensor, nn

from priml_b200.config import Fig

__all__ = ["Float8ModelQuantization", "NoModelQuantization"]

log = logging.getLogger(__name__)

_RECIPES = ("mxfp8", "tensorwise", "rowwise", "rowwise_gw_hp")
_CLASSES: dict[type, type] = {}


class NoModelQuantization:
    """No quantization (default)."""

    class Config(Fig["NoModelQuantization"]):
        pass

    def __init__(self, config: Config | None = None) -> None:
        del config

    def __call__(self, model: nn.Module) -> nn.Module:
        return model


def _mx_forward(self: nn.Linear, input: Tensor, *args: Any, **kwargs: Any) -> Tensor:  # noqa: A002
    del args, kwargs
    from priml_b200.ops.mx import mx_linear

    return mx_linear(input, self.weight, wgrad_high_precision=self._mx_wgrad_hp)


def _mx_class(cls: type) -> type:
    """``cls`` with an MXFP8 forward (one subclass per linear class)."""
    if cls not in _CLASSES:
        _CLASSES[cls] = type(f"MXFP8{cls.__name__}", (cls,), {"forward": _mx_forward, "__module__": __name__})
    return _CLASSES[cls]


class Float8ModelQuantization:
    """Convert selected linear layers to MXFP8 training."""

    class Config(Fig["Float8ModelQuantization"]):
        recipe: str = "mxfp8"
        """``mxfp8`` / ``tensorwise`` / ``rowwise`` (all GEMMs MXFP8) or ``rowwise_gw_hp`` (bf16 weight gradient)."""
        module_filter: Callable[[nn.Module, str], bool] | None = None
        """Optional filter ``(module, fqn) -> bool`` selecting the layers to convert."""
        enable_fsdp_float8_all_gather: bool = False
        """Accepted for config compatibility (see the module docstring)."""

    def __init__(self, config: Config | None = None) -> None:
        config = config or Float8ModelQuantization.Config()
        if config.recipe not in _RECIPES:
            raise ValueError(f"Invalid recipe {config.recipe!r}. Choose from: {list(_RECIPES)}")
        self.config = config
        self.module_filter = config.module_filter
        self.wgrad_hp = config.recipe == "rowwise_gw_hp"
        self.converted_count = 0
        self.enabled = True

    @staticmethod
    def _default_module_filter(mod: nn.Module, fqn: str) -> bool:
        del fqn
        if not isinstance(mod, nn.Linear) or mod.bias is not None:
            return False
        return mod.weight.shape[0] % 32 == 0 and mod.weight.shape[1] % 32 == 0

    def __call__(self, model: nn.Module) -> nn.Module:
        keep = self.module_filter or self._default_module_filter
        count = 0
        for name, mod in model.named_modules():
            if keep(mod, name) and not getattr(mod, "_mx_converted", False):
                mod.__class__ = _mx_class(type(mod))
                mod._mx_wgrad_hp = self.wgrad_hp  # noqa: SLF001
                mod._mx_converted = True  # noqa: SLF001
                count += 1
        self.converted_count = count
        log.info("Converted %d linear layers to MXFP8 (recipe=%s).", count, self.config.recipe)
        return model
