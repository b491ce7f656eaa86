"""NanoChat training step (``priml/baselines/nanochat/train_step.py:43-715``).

The recipe: NorMuon on the "reasoning" matrices and five AdamW members on the
rest, each at its own rate (tuned at width 768 and rescaled by
``1 / sqrt(width / 768)``), bf16 autocast, gradient accumulation up to a fixed
token batch, a trapezoidal learning-rate schedule and a weight-decay anneal
driven by the fraction of a wall-clock budget spent, a momentum ramp driven by
the step count, and a divergence guard that reads the loss only at an
accumulation boundary (so no pass stalls the host on the device).

The budget clock charges optimizer steps after ``budget_warmup_steps`` and is
bracketed by device synchronizations at accumulation boundaries only, like the
reference's. The loss is the fused soft-capped linear + cross-entropy of
:meth:`NanoChatLM.token_loss` (no ``[B, S, V]`` logits), in place of the
reference's compiled model + loss graph.
"""

from __future__ import annotations

import contextlib
import math
import time
from dataclasses import field
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.baselines.nanochat.model import NanoChatLM
from priml_b200.config import Makes, PartialConfig
from priml_b200.loss import TokenCrossEntropy
from priml_b200.math.schedules import trapezoidal
from priml_b200.optimizers import FusedAdamW, apply_lr_scale
from priml_b200.optimizers.composite import CompositeOptimizer, excluding, matching
from priml_b200.optimizers.muon import NorMuon
from priml_b200.train.train_step import TrainStep, TrainStepOutput

__all__ = ["NanoChatTrainStep", "matrix_parameters", "nanochat_loss", "nanochat_optimizer"]


def matrix_parameters() -> Any:
    """Rank >= 2 parameters that are not lookup tables (the orthogonalizing member's)."""
    return excluding(NorMuon.eligible_tensor, "embed", "lm_head")


def nanochat_loss() -> TokenCrossEntropy.Config:
    """Unreduced per-token CE over ``media`` / ``label`` batches (ignore index -1)."""
    return TokenCrossEntropy.Config(input_key="media", target_key="label", ignore_index=-1)


# Which members' rates scale with 1/sqrt(width): the two scalar groups step per-layer numbers, not matrices.
WIDTH_SCALED = (True, True, True, False, False, False)


def nanochat_optimizer(*, compile: bool = True) -> CompositeOptimizer.Config:  # noqa: A002
    """NorMuon on the reasoning matrices, AdamW on everything else, by class.

    Rates are stated as tuned at 768 channels; the step's ``finalize`` rescales
    the width-scaled members (:data:`WIDTH_SCALED`) to the model's width.
    """
    def adam(lr: float, betas: tuple[float, float] = (0.8, 0.95)) -> FusedAdamW.Config:
        return FusedAdamW.Config(lr=lr, betas=betas, eps=1e-10, weight_decay=0.0, compile=compile)

    config = CompositeOptimizer.Config()
    config.optimizers = [
        adam(0.004),  # unembedding
        adam(0.6),  # token embedding
        adam(0.6),  # value embeddings
        adam(0.5 * 0.01),  # residual mix (scales the whole stream)
        adam(0.5, (0.96, 0.95)),  # skip mix (starts at 0.1 and must travel)
        NorMuon.Config(compile=compile),
    ]
    # most specific first: ``value_embeds`` also contains ``embed``
    config.select = [
        matching("lm_head"),
        excluding(matching("embed"), "value_embeds"),
        matching("value_embeds"),
        matching("mix.running"),
        matching("mix.original"),
        matrix_parameters(),
    ]
    config.drop_empty = True
    return config


class NanoChatTrainStep(TrainStep):
    """Budgeted, accumulated, schedule-driven step of the nanochat recipe."""

    class Config(Makes["NanoChatTrainStep"], TrainStep.Config):
        model: Any = field(default_factory=NanoChatLM.Config)
        optimizer: Any = field(default_factory=nanochat_optimizer)
        loss: Any = field(default_factory=nanochat_loss)
        dtype_autocast: torch.dtype | None = torch.bfloat16
        train_budget_sec: float = 300.0
        """Training seconds the schedules anneal over (this step's own clock)."""
        schedule: Any = field(default_factory=lambda: PartialConfig(trapezoidal, flat=0.5))
        """Budget progress in [0, 1] -> learning-rate multiplier."""
        budget_warmup_steps: int = 11
        tokens_per_optimizer_step: int = 524_288
        rows_per_pass: int = 32
        momentum_start: float = 0.85
        momentum_end: float = 0.95
        momentum_warmup_steps: int = 300
        decay_to_zero: bool = True
        divergence_threshold: float = 100.0
        adam_lr_tuned_at_channels: int = 768
        width_scaled: tuple[bool, ...] = WIDTH_SCALED

        def finalize(self):  # noqa: ANN201
            if self.train_budget_sec <= 0 or not math.isfinite(self.train_budget_sec):
                raise ValueError(f"train_budget_sec must be finite and positive; got {self.train_budget_sec}.")
            if self.budget_warmup_steps < 0:
                raise ValueError(f"budget_warmup_steps must be nonnegative; got {self.budget_warmup_steps}.")
            if self.momentum_warmup_steps <= 0:
                raise ValueError(f"momentum_warmup_steps must be positive; got {self.momentum_warmup_steps}.")
            if self.rows_per_pass <= 0 or self.tokens_per_optimizer_step <= 0:
                raise ValueError("rows_per_pass and tokens_per_optimizer_step must be positive.")
            if math.isnan(self.gradient_clip_norm) or self.gradient_clip_norm <= 0:
                raise ValueError(f"gradient_clip_norm must be positive; got {self.gradient_clip_norm}.")
            if math.isnan(self.divergence_threshold) or self.divergence_threshold <= 0:
                raise ValueError(f"divergence_threshold must be positive; got {self.divergence_threshold}.")
            for name, m in (("momentum_start", self.momentum_start), ("momentum_end", self.momentum_end)):
                if math.isnan(m) or not 0.0 <= m < 1.0:
                    raise ValueError(f"{name} must lie in [0, 1); got {m}.")
            per_pass = self.rows_per_pass * self.model.max_seq_len
            if self.tokens_per_optimizer_step % per_pass:
                raise ValueError(
                    f"tokens_per_optimizer_step={self.tokens_per_optimizer_step} is not divisible by "
                    f"rows_per_pass * max_seq_len={per_pass}."
                )
            # rescale the width-scaled AdamW members once, then pin the tuned width to the model's
            if isinstance(self.optimizer, CompositeOptimizer.Config):
                width = self.model.channels_in
                for member, scaled in zip(self.optimizer.optimizers, self.width_scaled, strict=False):
                    if scaled and isinstance(member, FusedAdamW.Config):
                        member.lr = member.lr / math.sqrt(width / self.adam_lr_tuned_at_channels)
            self.adam_lr_tuned_at_channels = self.model.channels_in
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__(config)
        self.config: NanoChatTrainStep.Config = config
        self.accumulate_passes = config.tokens_per_optimizer_step // (config.rows_per_pass * config.model.max_seq_len)
        self.clock = _BudgetClock(config.budget_warmup_steps, self._synchronize)
        self.window = _PassWindow(self.accumulate_passes)
        self.lr_schedule = config.schedule.make()
        self.knobs = _RecipeKnobs(config)
        for group in self.optimizer.param_groups:
            group.setdefault("initial_weight_decay", group.get("weight_decay", 0.0))

    # The budget clock is the recipe's notion of time: schedules anneal over it and the loop's
    # time limit reads it.
    @property
    def elapsed_sec(self) -> float:
        return self.clock.seconds

    @elapsed_sec.setter
    def elapsed_sec(self, value: float) -> None:
        self.clock.seconds = float(value)

    @property
    def progress_learning_schedule(self) -> float:
        return min(self.clock.seconds / float(self.config.train_budget_sec), 1.0)

    @property
    def global_step(self) -> int:
        return int(self.timer_step.global_count)

    def _per_token_loss(self, batch: dict[str, Any]) -> Tensor:
        return self.compute_loss(**batch)["loss"]

    def train_step(self, **batch: Any) -> TrainStepOutput:  # type: ignore[override]
        """Forward + backward of one pass; the optimizer steps when the window of passes is full."""
        with self.clock.charge(boundary=self.window.empty):
            self.model.train()
            per_token = self._per_token_loss(batch)
            loss = per_token.float().mean()
            (loss / self.accumulate_passes).backward()
            self.window.add(loss.detach())
            metrics: dict[str, Any] = {}
            if self.window.full:
                with self.timer_step:
                    metrics = self._apply_update()
                self.clock.count_step()
                worst = self.window.close()
            else:
                worst = None
        if worst is not None:
            self._check_loss(worst)
        self.last_loss = loss.detach()
        stepped = self.window.empty
        return TrainStepOutput({"loss": loss.detach().reshape(1), "model": per_token.detach(), "metrics": metrics,
                                "num_samples": int(per_token.shape[0]), "stepped": stepped})  # fmt: skip

    def train_loss(self, **batch: Any) -> TrainStepOutput:
        self.model.train()
        with torch.no_grad():
            per_token = self._per_token_loss(batch)
        return TrainStepOutput({"loss": per_token.float().mean().reshape(1), "model": per_token})

    def eval_loss(self, **batch: Any) -> TrainStepOutput:
        """Mean over the real rows only (``valid_count``); ``model`` is the per-token loss."""
        self.model.eval()
        with torch.inference_mode():
            per_token = self._per_token_loss(batch)
        valid = int(batch.get("valid_count", per_token.shape[0]))
        return TrainStepOutput({"loss": per_token[:valid].float().mean().reshape(1), "model": per_token})

    def call_eval(self, *args: Any, **batch: Any) -> Tensor:
        self.model.eval()
        with torch.inference_mode(), self._autocast():
            return self.model(batch["media"])

    def on_epoch_end(self) -> None:
        """A partly filled window at the end of the data is discarded, gradients included."""
        if not self.window.empty:
            self.model.zero_grad(set_to_none=True)
            self.window.reset()

    def state_dict(self) -> dict[str, Any]:
        state = super().state_dict()
        state["elapsed_sec"] = self.clock.seconds
        state["local_step"] = self.clock.steps
        return state

    def load_state_dict(self, state_dict: dict[str, Any], **kwargs: Any) -> None:
        del kwargs
        if "local_step" not in state_dict:
            raise ValueError("checkpoint lacks 'local_step': the budget clock of that run cannot be resumed.")
        super().load_state_dict(state_dict)
        self.clock.seconds = float(state_dict["elapsed_sec"])
        self.clock.steps = int(state_dict["local_step"])
        self.window.reset()

    def charge_budget(self, seconds: float) -> None:
        """Bill loop-side work (fetching and staging a batch) to the budget, once warmup is over."""
        self.clock.bill(seconds)

    def _check_loss(self, worst: Tensor) -> None:
        """One host read per optimizer step: the worst pass loss of the window just closed."""
        value = float(worst)
        if math.isfinite(value) and value <= self.config.divergence_threshold:
            return
        self.model.zero_grad(set_to_none=True)
        self.window.reset()
        raise RuntimeError(f"loss {value} crossed the divergence limit at optimizer step {self.global_step}.")

    def _apply_update(self) -> dict[str, Any]:
        metrics: dict[str, Any] = {}
        if math.isfinite(self.config.gradient_clip_norm):
            norm = nn.utils.clip_grad_norm_(self.model.parameters(), self.config.gradient_clip_norm)
            metrics["grad_norm"] = norm.detach()
        progress = self.progress_learning_schedule
        apply_lr_scale([self.optimizer], float(self.lr_schedule(progress)))
        momentum = self.knobs.momentum(self.global_step)
        decay_scale = self.knobs.decay_scale(progress)
        for group in self.optimizer.param_groups:
            if "momentum" in group:
                group["momentum"] = momentum
            if "weight_decay" in group and decay_scale is not None:
                group["weight_decay"] = group["initial_weight_decay"] * decay_scale
        self.optimizer.step()
        self.model.zero_grad(set_to_none=True)
        metrics.update({f"lr_{name}": rate for name, rate in _learning_rates(self.optimizer).items()})
        metrics["progress"] = progress
        metrics["momentum"] = momentum
        return metrics

    def _synchronize(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize()


class _BudgetClock:
    """Seconds of training spent, counted only after ``warmup_steps`` optimizer steps.

    Passes are timed on the host; the device is synchronized only at the edges of a window of
    passes, so the charge for a window is exact while no single pass waits for the GPU.
    """

    def __init__(self, warmup_steps: int, synchronize: Any) -> None:
        self.warmup_steps = warmup_steps
        self.synchronize = synchronize
        self.seconds = 0.0
        self.steps = 0  # optimizer steps taken by this process

    @property
    def running(self) -> bool:
        return self.steps > self.warmup_steps

    def count_step(self) -> None:
        self.steps += 1

    def bill(self, seconds: float) -> None:
        if self.running:
            self.seconds += seconds

    @contextlib.contextmanager
    def charge(self, *, boundary: bool) -> Any:
        if boundary:
            self.synchronize()
        began = time.perf_counter()
        stepped_before = self.steps
        yield
        if self.running:
            if self.steps != stepped_before:
                self.synchronize()
            self.seconds += time.perf_counter() - began


class _PassWindow:
    """The passes of one optimizer step and the largest pass loss among them (kept on the device)."""

    def __init__(self, size: int) -> None:
        self.size = size
        self.count = 0
        self.worst: Tensor | None = None

    @property
    def empty(self) -> bool:
        return self.count == 0

    @property
    def full(self) -> bool:
        return self.count >= self.size

    def add(self, loss: Tensor) -> None:
        self.worst = loss if self.worst is None else torch.maximum(self.worst, loss)
        self.count += 1

    def close(self) -> Tensor | None:
        worst = self.worst
        self.reset()
        return worst

    def reset(self) -> None:
        self.count = 0
        self.worst = None


class _RecipeKnobs:
    """Momentum ramp over the first steps and weight-decay anneal over the budget."""

    def __init__(self, config: NanoChatTrainStep.Config) -> None:
        self.start, self.end = config.momentum_start, config.momentum_end
        self.ramp_steps = config.momentum_warmup_steps
        self.anneal_decay = config.decay_to_zero

    def momentum(self, step: int) -> float:
        ramp = min(step / self.ramp_steps, 1.0)
        return self.start + (self.end - self.start) * ramp

    def decay_scale(self, progress: float) -> float | None:
        return max(0.0, 1.0 - progress) if self.anneal_decay else None


def _learning_rates(optimizer: Any) -> dict[str, float]:
    """One rate per optimizer member, keyed by its lowercased class name."""
    if not isinstance(optimizer, CompositeOptimizer):
        return {"all": float(optimizer.param_groups[0]["lr"])}
    return {type(m).__name__.lower(): float(m.param_groups[0]["lr"]) for m in optimizer.optimizers if m.param_groups}

