"""Exponential moving average of weights (``priml/train/ema.py:21-547``).

The config fields, methods and the checkpoint layout are the reference's, so
recipes and checkpoints carry over between the two frameworks:

* ``EMA.Config``: ``decay``, ``update_after_step`` (calls that only count before
  averaging starts), ``update_every``, ``track_buffers``, ``shadow_kind``
  (``"module"``: a deep copy of the model; ``"param_dict"``: name-keyed clones of
  each parameter's local shard, which survive FSDP / DTensor sharding),
  ``warmup_seed`` and ``decay_schedule`` (``(decay, step) -> decay``).
* ``state_dict()``: ``global_step`` and ``local_step`` plus ``shadow_model`` (module
  shadows) or ``shadow_params`` / ``shadow_buffers`` (param_dict shadows).

The shadow is created on the first call from the model it is given. One
averaging step is a single multi-tensor lerp over every tracked tensor, so an
update costs a few fused kernel launches rather than two per parameter.
"""

from __future__ import annotations

import contextlib
import copy
from collections import OrderedDict
from collections.abc import Callable, Iterator
from typing import Any, Literal

import torch
from torch import Tensor, nn

from priml_b200.config import Fig

__all__ = ["EMA", "NoEMA", "constant_decay", "karras_decay"]


def constant_decay(decay: float, step: int) -> float:
    """The configured decay at every step."""
    del step
    return decay


def karras_decay(decay: float, step: int) -> float:
    """Decay that starts near 0.1 and rises as ``(1 + step) / (10 + step)``, never above ``decay``.

    Early averages then forget their first snapshots quickly (Karras et al. 2023,
    arXiv:2312.02696).
    """
    return min(decay, (1 + step) / (10 + step))


def _clone_state(source: Any) -> OrderedDict:
    """Detached copies of a state dict's tensors, keeping torch's version ``_metadata``."""
    out = OrderedDict((k, v.detach().clone() if torch.is_tensor(v) else v) for k, v in source.items())
    meta = getattr(source, "_metadata", None)
    if meta is not None:
        out._metadata = meta  # type: ignore[attr-defined]  # noqa: SLF001
    return out


class NoEMA:
    """Disabled averaging with the same surface as :class:`EMA` (the counters still checkpoint)."""

    class Config(Fig["NoEMA"]):
        pass

    def __init__(self, _config: Config | None = None) -> None:
        self.shadow_model: nn.Module | None = None
        self.global_step = 0
        self.local_step = 0

    def __call__(self, model: nn.Module) -> None:
        del model

    @contextlib.contextmanager
    def apply_to(self, model: nn.Module) -> Iterator[None]:
        del model
        yield

    def state_dict(self) -> dict[str, Any]:
        return {"global_step": self.global_step, "local_step": self.local_step}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        self.global_step = int(state_dict.get("global_step", 0))
        self.local_step = int(state_dict.get("local_step", 0))


class EMA:
    """Moving average of a model's trainable parameters (and, optionally, a copy of its buffers)."""

    class Config(Fig["EMA"]):
        decay: float = 0.9999
        """Weight of the old average in each update."""
        update_after_step: int = 0
        """Calls that only advance the counter; the first average happens at this call index."""
        update_every: int = 1
        """Average on every n-th call counted from ``update_after_step``."""
        track_buffers: bool = True
        """Copy non-parameter buffers into the shadow at each update."""
        shadow_kind: Literal["module", "param_dict"] = "module"
        """``"module"``: deep-copied model; ``"param_dict"``: clones of the local parameter shards."""
        warmup_seed: bool = False
        """At the first averaging call, copy the live weights instead of averaging."""
        decay_schedule: Callable[[float, int], float] = constant_decay
        """``(decay, averaging step) -> decay used at that step``."""

    def __init__(self, config: Config) -> None:
        if not 0.0 <= config.decay <= 1.0:
            raise ValueError(f"decay must lie in [0, 1]; got {config.decay}.")
        if config.update_every < 1:
            raise ValueError(f"update_every must be at least 1; got {config.update_every}.")
        if config.update_after_step < 0:
            raise ValueError(f"update_after_step must be non-negative; got {config.update_after_step}.")
        self.decay = config.decay
        self.update_after_step = config.update_after_step
        self.update_every = config.update_every
        self.track_buffers = config.track_buffers
        self.shadow_kind = config.shadow_kind
        self.warmup_seed = config.warmup_seed
        self.decay_schedule = config.decay_schedule
        self.shadow_model: nn.Module | None = None
        self.shadow_params: dict[str, Tensor] = {}
        self._shadow_buffers: dict[str, Tensor] = {}
        self._names: list[str] = []  # tracked parameter names, in model order
        self._filter: Callable[[str, nn.Parameter], bool] | None = None
        self._pending: dict[str, Any] | None = None  # a checkpoint read before the shadow existed
        self._backup: list[Tensor] = []
        self._ready = False  # the shadow exists (made from the model at the first update or swap)
        self.global_step = 0
        self.local_step = 0

    # ------------------------------------------------------------------ configuration
    def set_param_filter(self, param_filter: Callable[[str, nn.Parameter], bool] | None) -> None:
        """Track only the parameters the predicate accepts; call before the first update."""
        if self._ready:
            raise RuntimeError("set_param_filter must come before the first EMA update.")
        self._filter = param_filter

    def effective_decay(self, step: int) -> float:
        decay = self.decay_schedule(self.decay, step)
        if not 0.0 <= decay <= 1.0:
            raise ValueError(f"decay_schedule gave {decay} at step {step}; an average needs a value in [0, 1].")
        return decay

    # ------------------------------------------------------------------ shadow storage
    def _tracked(self, model: nn.Module) -> list[str]:
        keep = self._filter
        return [n for n, p in model.named_parameters() if p.requires_grad and (keep is None or keep(n, p))]

    def _shadow_tensors(self) -> list[Tensor]:
        if self.shadow_model is not None:
            own = dict(self.shadow_model.named_parameters())
            return [own[n].data for n in self._names]
        return [self.shadow_params[n] for n in self._names]

    def _setup(self, model: nn.Module) -> None:
        if self.shadow_kind == "module":
            self._names = self._tracked(model)
            self.shadow_model = copy.deepcopy(model).eval().requires_grad_(False)
            if self._pending is not None:
                self.shadow_model.load_state_dict(self._pending["shadow_model"])
        elif self.shadow_params:
            # restored from a checkpoint before the first update: keep the averages, move them
            # next to the live tensors (a rank-0 checkpoint loads onto rank 0's device everywhere)
            live = dict(model.named_parameters())
            self.shadow_params = {n: t.to(live[n].device) if n in live else t for n, t in self.shadow_params.items()}
            bufs = dict(model.named_buffers())
            self._shadow_buffers = {n: t.to(bufs[n].device) if n in bufs else t for n, t in self._shadow_buffers.items()}
            self._names = [n for n, _ in model.named_parameters() if n in self.shadow_params]
        else:
            self._names = self._tracked(model)
            live = dict(model.named_parameters())
            self.shadow_params = {n: live[n].detach().clone() for n in self._names}
            if self.track_buffers:
                self._shadow_buffers = {n: b.detach().clone() for n, b in model.named_buffers()}
        self._pending = None
        params = dict(model.named_parameters())
        self._backup = [torch.empty_like(params[n].data) for n in self._names]
        self._ready = True

    def _refresh_buffers(self, model: nn.Module) -> None:
        live = dict(model.named_buffers())
        targets = (
            dict(self.shadow_model.named_buffers()) if self.shadow_model is not None else self._shadow_buffers
        )
        for name, buf in targets.items():
            if name in live:
                buf.data.copy_(live[name].data)

    # ------------------------------------------------------------------ updates
    @torch.no_grad()
    def __call__(self, model: nn.Module) -> None:
        if not self._ready:
            self._setup(model)
        call = self.global_step
        self.global_step += 1
        if call < self.update_after_step or (call - self.update_after_step) % self.update_every:
            return
        live = dict(model.named_parameters())
        current = [live[n].data for n in self._names]
        shadow = self._shadow_tensors()
        if self.warmup_seed and call == self.update_after_step:
            torch._foreach_copy_(shadow, current)
        else:
            # shadow <- decay * shadow + (1 - decay) * live, one multi-tensor kernel
            torch._foreach_lerp_(shadow, current, 1.0 - self.effective_decay(self.local_step))
        if self.track_buffers:
            self._refresh_buffers(model)
        self.local_step += 1

    @contextlib.contextmanager
    def apply_to(self, model: nn.Module) -> Iterator[None]:
        """Evaluate ``model`` with the averaged parameters; its own weights come back on exit.

        Buffers keep their live values.
        """
        if not self._ready:
            self._setup(model)
        live = dict(model.named_parameters())
        missing = [n for n in self._names if n not in live]
        if missing:
            raise RuntimeError(f"EMA.apply_to: tracked parameters {missing[:3]} are not in the model.")
        current = [live[n].data for n in self._names]
        swapped = False
        try:
            with torch.no_grad():
                torch._foreach_copy_(self._backup, current)
                torch._foreach_copy_(current, self._shadow_tensors())
                swapped = True
            yield
        finally:
            if swapped:
                with torch.no_grad():
                    torch._foreach_copy_(current, self._backup)

    # ------------------------------------------------------------------ checkpoints
    def state_dict(self) -> dict[str, Any]:
        counters = {"global_step": self.global_step, "local_step": self.local_step}
        if self.shadow_model is not None:
            return {"shadow_model": _clone_state(self.shadow_model.state_dict()), **counters}
        if not self._ready:
            return counters
        return {
            "shadow_params": {n: t.detach().clone() for n, t in self.shadow_params.items()},
            "shadow_buffers": {n: t.detach().clone() for n, t in self._shadow_buffers.items()},
            **counters,
        }

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        self.global_step = int(state_dict["global_step"])
        self.local_step = int(state_dict.get("local_step", 0))  # a step schedule resumes where it was
        if "shadow_model" in state_dict:
            saved = _clone_state(state_dict["shadow_model"])
            if self.shadow_model is None:
                self._pending = {"shadow_model": saved}
            else:
                self.shadow_model.load_state_dict(saved)
        elif "shadow_params" in state_dict:
            params = {n: t.detach().clone() for n, t in state_dict["shadow_params"].items()}
            buffers = {n: t.detach().clone() for n, t in state_dict.get("shadow_buffers", {}).items()}
            if not self._ready:
                # adopted as is: the averages are readable right after the load
                self.shadow_params, self._shadow_buffers = params, buffers
            else:
                for n, t in params.items():
                    self.shadow_params[n].copy_(t)
                for n, t in buffers.items():
                    self._shadow_buffers[n].copy_(t)
