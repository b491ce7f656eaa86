"""One optimization step over a model (``priml/train/train_step.py:63-828``).

Build order matches the reference: model (eager or on ``meta``) -> model
quantization -> parallel strategy (shard + materialize) -> activation strategy
-> optimizer (given the MODULE, falling back to its parameters) -> LR schedule
-> EMA. ``train_step(**batch)`` runs forward/loss/backward and, when the
accumulation window is complete, clip -> LR -> optimizer -> zero -> EMA.

B200 specifics:

* ``compile`` defaults to ``None`` (eager): the hot ops are hand-written kernels.
* For language models (``TokenCrossEntropy`` loss and a model with
  ``token_loss``) the loss runs fused from hidden states; logits never exist.
* Gradient clipping on CUDA with :class:`FusedAdamW` is device-side: the global
  norm and clip coefficient are computed by one multi-tensor kernel and folded
  into the optimizer kernel as a gradient scale -- no host synchronization.
* ``last_loss`` / ``last_grad_norm`` are device tensors; reading them is the
  caller's (one) sync point per step.
"""

from __future__ import annotations

import contextlib
import math
from collections.abc import Callable, Mapping
from dataclasses import field
from typing import Any, Literal

import torch
import torch.distributed as dist
from torch import Tensor, nn

from priml_b200.timer import CheckpointableStepTimer
from priml_b200.train.ema import NoEMA
from priml_b200.config import Fig, PartialConfig
from priml_b200.loss import SimpleLoss, TokenCrossEntropy
from priml_b200.math.schedules import constant
from priml_b200.models.special import Identity

__all__ = ["TrainStep", "TrainStepOutput"]


class TrainStepOutput(dict):
    """``{"loss": Tensor, "num_samples": int, "stepped": bool, ...}``."""


class _NoQuant:
    class Config(Fig["_NoQuant"]):
        pass

    def __init__(self, config: Any = None) -> None:
        del config

    def __call__(self, model: nn.Module) -> nn.Module:
        return model


class TrainStep:
    class Config(Fig["TrainStep"], kw_only=False):
        model: Any = field(default_factory=Identity.Config)
        optimizer: Any = field(
            default_factory=lambda: PartialConfig(torch.optim.AdamW, lr=1e-3, betas=(0.9, 0.999), weight_decay=1e-2)
        )
        loss: Any = field(default_factory=SimpleLoss.Config)
        accumulate_grad_batches: int = 1
        drop_partial_accumulation_on_epoch_end: bool = True
        train_budget_steps: float = math.inf
        train_budget_sec: float = math.inf
        train_budget_epochs: float = math.inf
        learning_rate_scheduler: Any = field(default_factory=lambda: PartialConfig(constant))
        parallelism: Any = None
        """Placement / sharding strategy; ``None`` = ``NoParallel`` on the default device."""
        model_quantization: Any = field(default_factory=_NoQuant.Config)
        activation_memoization: Any = None
        compile: Any = None
        ema: Any = field(default_factory=lambda: NoEMA.Config())
        gradient_clip_norm: float = math.inf
        device_init: Literal["meta", "eager"] = "eager"
        dtype_autocast: torch.dtype | None = None
        autocast_cache_enabled: bool = False

    def __init__(self, config: Config) -> None:
        from priml_b200.parallel.strategies import NoParallel

        self.config = config
        ctx = torch.device("meta") if config.device_init == "meta" else contextlib.nullcontext()
        with ctx:
            model = config.model.make()
        model = config.model_quantization.make()(model)
        strategy = config.parallelism.make() if config.parallelism is not None else NoParallel()
        self.parallelism = strategy
        model = strategy(model)
        if config.activation_memoization is not None:
            model = config.activation_memoization.make()(model)
        self.model: nn.Module = model
        self.device = next((p.device for p in model.parameters()), getattr(strategy, "device", torch.device("cpu")))
        if hasattr(strategy, "build_optimizer"):
            self.optimizer = strategy.build_optimizer(config.optimizer.make(), model)
        else:
            self.optimizer = self.build_optimizer(model)
        for g in self.optimizer.param_groups:
            g.setdefault("initial_lr", g["lr"])
        self.schedule: Callable[[float], float] = config.learning_rate_scheduler.make()
        self.ema = config.ema.make() if config.ema is not None else NoEMA()
        self.loss_fn = config.loss.make()
        self._compiled: Callable[..., Any] | None = None
        self.accumulation_steps = 0
        self.accumulated_samples = 0
        self.timer_forward = CheckpointableStepTimer()
        self.timer_eval = CheckpointableStepTimer()
        self.timer_step = CheckpointableStepTimer()
        self.epoch = 0.0
        self.epoch_timer: Any = None
        self.last_loss: Tensor | None = None
        self.last_grad_norm: Tensor | None = None
        self._grad_params: list[Tensor] = [p for p in model.parameters() if p.requires_grad]

    # ------------------------------------------------------------------ construction
    def build_optimizer(self, model: nn.Module) -> torch.optim.Optimizer:
        make = self.config.optimizer.make()
        try:
            opt = make(model)
            if isinstance(opt, torch.optim.Optimizer):
                return opt
        except (TypeError, AttributeError, ValueError):
            pass
        return make([p for p in model.parameters() if p.requires_grad])

    def bind_epoch_timer(self, timer: Any) -> None:
        self.epoch_timer = timer

    # ------------------------------------------------------------------ progress
    def progress_complete(self) -> float:
        """Fraction of the tightest budget spent (steps, seconds or epochs)."""
        c = self.config
        fr = 0.0
        if math.isfinite(c.train_budget_steps):
            fr = max(fr, self.timer_step.global_count / max(1.0, c.train_budget_steps))
        if math.isfinite(c.train_budget_sec):
            fr = max(fr, self.timer_step.global_sec / max(1e-9, c.train_budget_sec))
        if math.isfinite(c.train_budget_epochs):
            ep = self.epoch_timer.epoch if self.epoch_timer is not None else self.epoch
            fr = max(fr, ep / max(1e-9, c.train_budget_epochs))
        return min(1.0, fr)

    def apply_learning_rate(self) -> float:
        scale = float(self.schedule(self.progress_complete()))
        for g in self.optimizer.param_groups:
            g["lr"] = g.get("initial_lr", g["lr"]) * scale
        return scale

    # ------------------------------------------------------------------ batches
    def preprocess_batch(self, batch: dict[str, Any]) -> dict[str, Any]:
        """Host -> device copy (``non_blocking`` from pinned memory)."""
        dev = self.device
        out = {}
        for k, v in batch.items():
            out[k] = v.to(dev, non_blocking=True) if isinstance(v, Tensor) and v.device != dev else v
        return out

    def _autocast(self) -> Any:
        dt = self.config.dtype_autocast
        if dt is None:
            return contextlib.nullcontext()
        return torch.autocast(self.device.type, dtype=dt, cache_enabled=self.config.autocast_cache_enabled)

    def __call__(self, **batch: Any) -> Any:
        fn: Callable[..., Any] = self.model
        if self.config.compile is not None:
            if self._compiled is None:
                self._compiled = self.config.compile.make()(self.model)
            fn = self._compiled
        with self._autocast():
            if "media" in batch:
                return fn(batch["media"])
            if "tokens" in batch:
                return fn(batch["tokens"])
            return fn(**batch)

    def compute_loss(self, **batch: Any) -> dict[str, Tensor]:
        if isinstance(self.loss_fn, TokenCrossEntropy) and hasattr(self.model, "token_loss"):
            with self._autocast():
                return self.loss_fn.fused(self.model, **batch)
        out = self(**batch)
        with self._autocast():
            return self.loss_fn(out, **batch)

    def _forward(self, batch: dict[str, Any]) -> Any:
        if "media" in batch:
            return self.model(batch["media"])
        if "tokens" in batch:
            return self.model(batch["tokens"])
        return self.model(**batch)

    def call_eval(self, *args: Any, **batch: Any) -> Any:
        """Model output in eval mode under ``inference_mode``, autocast and the EMA
        weights (``ema.apply_to``); the previous train/eval mode is restored."""
        was_training = self.model.training
        self.model.eval()
        try:
            with self.timer_eval, torch.inference_mode(), self.ema.apply_to(self.model), self._autocast():
                return self.model(*args, **batch) if args else self._forward(batch)
        finally:
            self.model.train(was_training)

    def _loss_from(self, output: Any, batch: dict[str, Any]) -> dict[str, Any]:
        with self._autocast():
            result = dict(self.loss_fn(output, **batch))
        result["model"] = output
        return result

    def train_loss(self, **batch: Any) -> TrainStepOutput:
        """Loss in train mode, without backprop."""
        with torch.no_grad():
            if isinstance(self.loss_fn, TokenCrossEntropy) and hasattr(self.model, "token_loss"):
                self.model.train()
                return TrainStepOutput(self.compute_loss(**batch))
            return TrainStepOutput(self._loss_from(self(**batch), batch))

    def eval_loss(self, **batch: Any) -> TrainStepOutput:
        """Loss in eval mode with the EMA weights (the evaluation path of the train loop)."""
        if isinstance(self.loss_fn, TokenCrossEntropy) and hasattr(self.model, "token_loss"):
            was_training = self.model.training
            self.model.eval()
            try:
                with self.timer_eval, torch.inference_mode(), self.ema.apply_to(self.model), self._autocast():
                    return TrainStepOutput(self.loss_fn.fused(self.model, **batch))
            finally:
                self.model.train(was_training)
        return TrainStepOutput(self._loss_from(self.call_eval(**batch), batch))

    # ------------------------------------------------------------------ update
    def _clip(self) -> Tensor | None:
        c = self.config.gradient_clip_norm
        if hasattr(self.optimizer, "fused_grad_norm"):
            if math.isinf(c):
                self.optimizer.grad_scale = None
                return None
            from priml_b200.train.grad_clip import fused_grad_norm_clip

            res = fused_grad_norm_clip(self.optimizer, c)
            if res is not None:
                norm, clip = res
                self.optimizer.grad_scale = clip
                return norm
        if math.isinf(c):
            return None
        return torch.nn.utils.clip_grad_norm_(self._grad_params, c)

    def step(self) -> None:
        """clip -> schedule -> optimizer.step -> zero_grad -> EMA."""
        with self.timer_step:
            self.last_grad_norm = self._clip()
            self.apply_learning_rate()
            self.optimizer.step()
            self.optimizer.zero_grad(set_to_none=True)
            self.ema(self.model)

    def train_step(self, **batch: Any) -> TrainStepOutput:
        """Forward + backward on one micro-batch; steps when the window closes."""
        sync = getattr(self.model, "set_requires_gradient_sync", None)
        if callable(sync) and self.config.accumulate_grad_batches > 1:
            sync(self.accumulation_steps + 1 >= self.config.accumulate_grad_batches)
        with self.timer_forward:
            losses = self.compute_loss(**batch)
            loss = losses["loss"]
            n = int(loss.shape[0]) if loss.ndim > 0 else 1
            total = loss.float().sum()
            if self.config.accumulate_grad_batches > 1:
                total = total / self.config.accumulate_grad_batches
            denom = loss.numel() if loss.ndim > 0 else 1
            (total / denom).backward()
        self.accumulation_steps += 1
        self.accumulated_samples += n
        stepped = False
        if self.accumulation_steps >= self.config.accumulate_grad_batches:
            self._assert_uniform_microbatch_count()
            self.step()
            self.accumulation_steps = 0
            self.accumulated_samples = 0
            stepped = True
        self.last_loss = loss.detach().float().mean()
        # Like the reference: the unreduced loss (and every other loss term) is returned;
        # ``last_loss`` holds the scalar mean for logging.
        out = TrainStepOutput({k: (v.detach() if isinstance(v, Tensor) else v) for k, v in losses.items()})
        out["num_samples"] = n
        out["stepped"] = stepped
        return out

    def on_epoch_end(self) -> None:
        self.epoch += 1
        if self.config.drop_partial_accumulation_on_epoch_end and self.accumulation_steps:
            self.optimizer.zero_grad(set_to_none=True)
            self.accumulation_steps = 0
            self.accumulated_samples = 0

    def _assert_uniform_microbatch_count(self) -> None:
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
            return
        if self.config.accumulate_grad_batches == 1:
            return
        dev = self.device if self.device.type == "cuda" else torch.device("cpu")
        t = torch.tensor([self.accumulation_steps, -self.accumulation_steps], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if int(t[0]) != -int(t[1]):
            raise RuntimeError("ranks disagree on the number of accumulated micro-batches")

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict[str, Any]:
        return {
            "model": self.model.state_dict(),
            "optimizer": self.optimizer.state_dict(),
            "timer_forward": self.timer_forward.state_dict(),
            "timer_eval": self.timer_eval.state_dict(),
            "timer_step": self.timer_step.state_dict(),
            "ema": self.ema.state_dict(),
            "accumulation_steps": self.accumulation_steps,
            "accumulated_samples": self.accumulated_samples,
        }

    def load_state_dict(
        self,
        state_dict: dict[str, Any],
        *,
        strict: bool = True,
        load_optimizer: bool = True,
        remap: Callable[[Mapping[str, Any]], Mapping[str, Any]] | None = None,
    ) -> None:
        """Resume from a checkpoint (``priml/train/train_step.py:704-752`` semantics).

        ``remap`` rewrites the saved model keys first; ``strict`` requires an exact key match;
        ``load_optimizer=False`` keeps the fresh optimizer and EMA (fine-tuning a changed
        model). Timers absent from the checkpoint stay at zero. A pending gradient
        accumulation is not resumable, so the accumulation counters restart at zero.
        """
        model_state = state_dict["model"]
        if remap is not None:
            model_state = remap(model_state)
        self.model.load_state_dict(model_state, strict=strict)
        for name in ("timer_forward", "timer_eval", "timer_step"):
            if name in state_dict:
                getattr(self, name).load_state_dict(state_dict[name])
        self.accumulation_steps = 0
        self.accumulated_samples = 0
        if load_optimizer:
            self.optimizer.load_state_dict(state_dict["optimizer"])
            if "ema" in state_dict:
                self.ema.load_state_dict(state_dict["ema"])
