"""CIFAR-10 training step (``priml/baselines/cifar10/train_step.py:40-337``).

Augment on the device (reflect-pad + random crop + flip + optional cutout in
one fused kernel, ``ops/csrc/augment.cu``), forward under autocast in
channels-last, label-smoothed cross-entropy, clip, schedule, step. A
whitening layer is fitted from the first training batch (optionally cached to
a file). The learning rate follows ``schedule(progress)`` times a warmup of
``int(warmup_fraction * total_train_steps)`` whole steps. ``use_tta`` averages
logits over the image, two one-pixel-shifted reflect-padded crops, and the
mirror of each (six passes).
"""

from __future__ import annotations

import math
from dataclasses import field
from pathlib import Path
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from priml_b200.baselines.cifar10.model import ResNet
from priml_b200.config import Makes, PartialConfig
from priml_b200.data.augmentation_gpu import pad_crop_flip
from priml_b200.math.schedules import cosine
from priml_b200.optimizers import apply_lr_scale
from priml_b200.optimizers.composite import CompositeOptimizer
from priml_b200.train.train_step import TrainStep, TrainStepOutput

__all__ = ["Cifar10TrainStep", "tta_logits"]


def tta_logits(model: nn.Module, media: Tensor) -> Tensor:
    """Mean logits over the image and two shifted crops, each with its mirror."""
    def mirrored(view: Tensor) -> Tensor:
        return 0.5 * (model(view) + model(view.flip(-1)))

    size = media.shape[-1]
    padded = F.pad(media, (1,) * 4, "reflect")
    return (mirrored(media) + mirrored(padded[..., 0:size, 0:size]) + mirrored(padded[..., 2 : size + 2, 2 : size + 2])) / 3


class Cifar10TrainStep(TrainStep):
    class Config(Makes["Cifar10TrainStep"], TrainStep.Config):
        model: Any = field(default_factory=ResNet.Config)
        optimizer: Any = field(
            default_factory=lambda: CompositeOptimizer.Config(
                optimizers=[PartialConfig(torch.optim.AdamW, lr=1e-3, betas=(0.9, 0.999), weight_decay=5e-2)]
            )
        )
        total_train_steps: int = 4_000
        schedule: Any = field(default_factory=lambda: PartialConfig(cosine))
        warmup_fraction: float = 0.02
        label_smoothing: float = 0.1
        translate_pad: int = 4
        cutout_size: int = 0
        derandomized_flip: bool = False
        """Flip every image on odd steps and none on even, instead of at random."""
        use_tta: bool = False
        whiten_num_images: int = 5_000
        whiten_cache_path: str = ""

        def finalize(self):  # noqa: ANN201
            if not 0 <= self.warmup_fraction < 1:
                raise ValueError(f"warmup_fraction must be in [0, 1); got {self.warmup_fraction}.")
            return super().finalize()

    def __init__(self, config: Config) -> None:
        if config.total_train_steps <= 0:
            raise ValueError(f"total_train_steps must be positive; got {config.total_train_steps}.")
        super().__init__(config)
        self.config: Cifar10TrainStep.Config = config
        self.model.to(memory_format=torch.channels_last)
        self.lr_schedule = config.schedule.make()
        self._whitened = not hasattr(self.model, "init_whiten")

    @property
    def global_step(self) -> int:
        return int(self.timer_step.global_count)

    @property
    def progress_learning_schedule(self) -> float:
        return min(1.0, self.global_step / self.config.total_train_steps)

    def train_step(self, **batch: Any) -> TrainStepOutput:  # type: ignore[override]
        media, label = batch["media"], batch["label"]
        self._maybe_init_whiten(media)
        media = self._augment(media)
        self.model.train()
        with self._autocast():
            logits = self.model(media)
            loss = self._loss(logits, label)
        loss.sum().backward()
        if math.isfinite(self.config.gradient_clip_norm):
            nn.utils.clip_grad_norm_(self.model.parameters(), self.config.gradient_clip_norm)
        with self.timer_step:
            self._apply_schedule()
            self.optimizer.step()
            self.model.zero_grad(set_to_none=True)
        self.last_loss = loss.detach().mean()
        return TrainStepOutput({"loss": loss.detach(), "model": logits.detach(), "num_samples": int(label.shape[0]),
                                "stepped": True})  # fmt: skip

    def train_loss(self, **batch: Any) -> TrainStepOutput:
        self.model.train()
        with torch.no_grad(), self._autocast():
            logits = self.model(batch["media"])
            return TrainStepOutput({"loss": self._loss(logits, batch["label"]), "model": logits})

    def eval_loss(self, **batch: Any) -> TrainStepOutput:
        logits = self.call_eval(media=batch["media"])
        return TrainStepOutput({"loss": self._loss(logits, batch["label"]), "model": logits})

    def call_eval(self, *args: Any, **batch: Any) -> Tensor:
        media = args[0] if args else batch["media"]
        self.model.eval()
        with torch.inference_mode(), self._autocast():
            return tta_logits(self.model, media) if self.config.use_tta else self.model(media)

    def on_epoch_end(self) -> None:
        """Nothing accumulates across an epoch boundary."""

    def state_dict(self) -> dict[str, Any]:
        state = super().state_dict()
        state["whitened"] = self._whitened
        return state

    def load_state_dict(self, state_dict: dict[str, Any], **kwargs: Any) -> None:
        del kwargs
        super().load_state_dict(state_dict)
        self._whitened = bool(state_dict["whitened"])

    def _apply_schedule(self) -> None:
        c = self.config
        multiplier = float(self.lr_schedule(self.progress_learning_schedule))
        warmup = int(c.warmup_fraction * c.total_train_steps)
        if warmup and self.global_step < warmup:
            multiplier *= (self.global_step + 1) / warmup
        apply_lr_scale([self.optimizer], multiplier)

    def _augment(self, media: Tensor) -> Tensor:
        c = self.config
        flip = (self.global_step % 2 == 1) if c.derandomized_flip else None
        return pad_crop_flip(media, media.shape[-1], pad=c.translate_pad, flip=flip, cutout_size=c.cutout_size)

    def _loss(self, logits: Tensor, label: Tensor) -> Tensor:
        return F.cross_entropy(logits.float(), label, label_smoothing=self.config.label_smoothing, reduction="none")

    def _maybe_init_whiten(self, media: Tensor) -> None:
        if self._whitened:
            return
        model: Any = self.model
        cache = Path(self.config.whiten_cache_path) if self.config.whiten_cache_path else None
        if cache is not None and cache.is_file():
            model.whiten.weight.data.copy_(torch.load(cache, map_location=self.device, weights_only=True))
        else:
            model.init_whiten(media[: self.config.whiten_num_images])
            if cache is not None:
                cache.parent.mkdir(parents=True, exist_ok=True)
                torch.save(model.whiten.weight.data, cache)
        self._whitened = True
