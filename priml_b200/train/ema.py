"""Exponential moving average of weights (``priml/train/ema.py:21-547``).

``kind="param_dict"`` keeps fp32 clones of each parameter's LOCAL shard, so it
works unchanged under FSDP / TP; ``kind="module"`` deep-copies the model.
Supports warmup, ``update_every``, constant or Karras (power-law) decay, and
``apply_to`` swaps the averaged weights in for evaluation.
"""

from __future__ import annotations

import contextlib
import copy
from collections.abc import Iterator
from typing import Any, Literal

import torch
from torch import Tensor, nn

from priml_b200.config import Fig

__all__ = ["EMA", "NoEMA", "karras_decay"]


def _local(t: Tensor) -> Tensor:
    return t._local_tensor if hasattr(t, "_local_tensor") else t  # noqa: SLF001


def karras_decay(step: int, gamma: float = 6.94) -> float:
    """Power-function EMA profile (Karras et al. 2024): ``(1 - 1/t) ** (gamma + 1)``."""
    if step <= 0:
        return 0.0
    return (1.0 - 1.0 / step) ** (gamma + 1.0)


class NoEMA:
    class Config(Fig["Callable[..., NoEMA]"]):
        def make(self) -> Any:
            return lambda model: NoEMA()

    def __call__(self, model: nn.Module) -> None:
        del model

    @contextlib.contextmanager
    def apply_to(self, model: nn.Module) -> Iterator[None]:
        del model
        yield

    def state_dict(self) -> dict[str, Any]:
        return {}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        del s


class EMA:
    class Config(Fig["Callable[..., EMA]"]):
        decay: float = 0.999
        kind: Literal["param_dict", "module"] = "param_dict"
        warmup_steps: int = 0
        update_every: int = 1
        schedule: Literal["constant", "karras"] = "constant"
        karras_gamma: float = 6.94

        def make(self) -> Any:
            cfg = self.copy_tree().finalize()
            return lambda model: EMA(cfg, model)

    def __init__(self, config: Config, model: nn.Module) -> None:
        self.config = config
        self.step = 0
        self.module: nn.Module | None = None
        self.shadow: dict[str, Tensor] = {}
        if config.kind == "module":
            self.module = copy.deepcopy(model).eval()
            for p in self.module.parameters():
                p.requires_grad_(False)
        else:
            self.shadow = {n: _local(p).detach().float().clone() for n, p in model.named_parameters()}

    def _decay(self) -> float:
        c = self.config
        if self.step <= c.warmup_steps:
            return 0.0
        if c.schedule == "karras":
            return karras_decay(self.step - c.warmup_steps, c.karras_gamma)
        return c.decay

    @torch.no_grad()
    def __call__(self, model: nn.Module) -> None:
        self.step += 1
        if self.step % self.config.update_every:
            return
        d = self._decay()
        if self.module is not None:
            for s, p in zip(self.module.parameters(), model.parameters(), strict=True):
                _local(s).lerp_(_local(p).to(s.dtype), 1.0 - d)
            return
        for n, p in model.named_parameters():
            self.shadow[n].lerp_(_local(p).float(), 1.0 - d)

    @contextlib.contextmanager
    def apply_to(self, model: nn.Module) -> Iterator[None]:
        """Temporarily swap the averaged weights into ``model``."""
        saved = {n: _local(p).detach().clone() for n, p in model.named_parameters()}
        src = dict(self.module.named_parameters()) if self.module is not None else self.shadow
        with torch.no_grad():
            for n, p in model.named_parameters():
                _local(p).copy_(_local(src[n]).to(p.dtype))
        try:
            yield
        finally:
            with torch.no_grad():
                for n, p in model.named_parameters():
                    _local(p).copy_(saved[n])

    def state_dict(self) -> dict[str, Any]:
        if self.module is not None:
            return {"step": self.step, "module": self.module.state_dict()}
        return {"step": self.step, "shadow": dict(self.shadow)}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.step = int(s.get("step", 0))
        if self.module is not None and "module" in s:
            self.module.load_state_dict(s["module"])
        elif "shadow" in s:
            for k, v in s["shadow"].items():
                if k in self.shadow:
                    self.shadow[k].copy_(v)
