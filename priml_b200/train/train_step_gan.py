"""Two-player GAN step (``priml/train/train_step_gan.py:24-285``).

Each call runs ``n_discriminator_steps`` discriminator updates on
``cat(real, G(z).detach())`` with labels 1 / 0, then one generator update
whose loss scores ``D(G(z))`` through the discriminator's activations while
the discriminator's parameters are frozen (their prior ``requires_grad``
flags are restored afterwards, so intentionally frozen parameters stay frozen).
The discriminator's logging loss is accumulated on device and read once.
"""

from __future__ import annotations

from dataclasses import field
from typing import Any

import torch
from torch import Tensor

from priml_b200.config import Fig, Makeable, PartialConfig
from priml_b200.loss import AdversarialLoss
from priml_b200.math.schedules import staircase
from priml_b200.models.special import Identity
from priml_b200.train.train_step import TrainStep, TrainStepOutput

__all__ = ["GANTrainStep"]


def _player(loss: Any = None) -> TrainStep.Config:
    cfg = TrainStep.Config(
        model=Identity.Config(),
        optimizer=PartialConfig(torch.optim.Adam, lr=2e-4, betas=(0.5, 0.999)),
        train_budget_steps=400,
        learning_rate_scheduler=PartialConfig(staircase, gamma=0.5),
    )
    if loss is not None:
        cfg.loss = loss
    return cfg


class GANTrainStep:
    class Config(Fig["GANTrainStep"]):
        generator: Makeable[TrainStep] = field(default_factory=lambda: _player(AdversarialLoss.Config()))
        discriminator: Makeable[TrainStep] = field(default_factory=_player)
        n_discriminator_steps: int = 1

    def __init__(self, config: Config) -> None:
        if config.n_discriminator_steps <= 0:
            raise ValueError(f"n_discriminator_steps must be positive, got {config.n_discriminator_steps}")
        self.generator = config.generator.make()
        self.discriminator = config.discriminator.make()
        self.n_discriminator_steps = config.n_discriminator_steps
        self.global_step = 0
        self.local_step = 0

    def preprocess_batch(self, batch: dict[str, Any]) -> dict[str, Any]:
        return self.generator.preprocess_batch(batch)

    def call_eval(self, **kwargs: Any) -> Any:
        return self.generator.call_eval(**kwargs)

    def on_epoch_end(self) -> None:
        self.generator.on_epoch_end()
        self.discriminator.on_epoch_end()

    @staticmethod
    def _labels(n: int, device: torch.device) -> Tensor:
        return torch.cat([torch.ones(n, 1, device=device), torch.zeros(n, 1, device=device)])

    def _discriminator_loss_sum(self, real: Tensor, batch: dict[str, Any], mode: str) -> float:
        total: Tensor | None = None
        for _ in range(self.n_discriminator_steps):
            if mode == "train":
                with torch.no_grad():
                    fake = self.generator.model(**batch)
            else:
                fake = self.generator.call_eval(**batch)
            media = torch.cat([real, fake.detach()], dim=0)
            labels = self._labels(real.shape[0], media.device)
            fn = {"train": self.discriminator.train_step, "train_loss": self.discriminator.train_loss,
                  "eval": self.discriminator.eval_loss}[mode]  # fmt: skip
            step_loss = fn(media=media, label=labels)["loss"].detach().sum()
            total = step_loss if total is None else total + step_loss
        return float(total) if total is not None else 0.0

    def _combine(self, g: Any, d_sum: float, n: int, fake: Tensor) -> TrainStepOutput:
        out = TrainStepOutput(dict(g))
        out["loss"] = g["loss"] + d_sum / (self.n_discriminator_steps * n * 2)
        out["model"] = fake
        return out

    def train_step(self, *, media: Tensor, **batch: Any) -> TrainStepOutput:
        d_sum = self._discriminator_loss_sum(media, batch, "train")
        flags = {n: p.requires_grad for n, p in self.discriminator.model.named_parameters()}
        self.discriminator.model.requires_grad_(False)
        try:
            fake = self.generator.model(**batch)
            logits = self.discriminator.model(fake)
            g = self.generator.train_step(fake_logits=logits, fake_media=fake, real_media=media, **batch)
        finally:
            for n, p in self.discriminator.model.named_parameters():
                p.requires_grad_(flags[n])
        self.global_step += 1
        self.local_step += 1
        return self._combine(g, d_sum, media.shape[0], fake)

    def train_loss(self, *, media: Tensor, **batch: Any) -> TrainStepOutput:
        d_sum = self._discriminator_loss_sum(media, batch, "train_loss")
        fake = self.generator.model(**batch)
        logits = self.discriminator.model(fake)
        g = self.generator.train_loss(fake_logits=logits, fake_media=fake, real_media=media, **batch)
        return self._combine(g, d_sum, media.shape[0], fake)

    def eval_loss(self, *, media: Tensor, **batch: Any) -> TrainStepOutput:
        d_sum = self._discriminator_loss_sum(media, batch, "eval")
        fake = self.generator.call_eval(**batch)
        logits = self.discriminator.call_eval(media=fake)
        g = self.generator.eval_loss(fake_logits=logits, fake_media=fake, real_media=media, **batch)
        return self._combine(g, d_sum, media.shape[0], fake)

    def state_dict(self) -> dict[str, Any]:
        return {"generator": self.generator.state_dict(), "discriminator": self.discriminator.state_dict(),
                "global_step": self.global_step}  # fmt: skip

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.generator.load_state_dict(state["generator"])
        self.discriminator.load_state_dict(state["discriminator"])
        self.global_step = state["global_step"]
        self.local_step = 0
