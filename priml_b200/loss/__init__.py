"""Losses returning ``{"loss": unreduced tensor, ...}`` dicts (``priml/loss/``).

``TokenCrossEntropy`` is the LM loss. When the model exposes ``token_loss``
(``CausalLM``), :class:`priml_b200.train.TrainStep` calls it directly so the
logits are never materialized in fp32 (fused linear + CE on CUDA).
"""

from __future__ import annotations

import functools
import math
from collections.abc import Callable
from dataclasses import field
from typing import Any, Protocol

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200 import ops
from priml_b200.config import Fig

__all__ = [
    "AdversarialLoss",
    "ClippedPolicyLoss",
    "DiffusionLoss",
    "LPIPS",
    "LPIPSLoss",
    "LossOutput",
    "SimpleLoss",
    "SimpleLossFn",
    "TokenCrossEntropy",
    "WeightedSum",
    "categorical_entropy",
    "clipped_policy_loss",
]

LossOutput = dict[str, Tensor]



class SimpleLossFn(Protocol):
    """A PyTorch-style loss function: ``fn(input, target, reduction=...)``."""

    def __call__(self, input: Tensor, target: Tensor, *, reduction: str = "mean") -> Tensor: ...  # noqa: A002

class SimpleLoss:
    """Wraps a functional loss: ``{"loss": loss_fn(prediction, batch[target_key], **kwargs)}``."""

    class Config(Fig["SimpleLoss"]):
        loss_fn: Callable[..., Tensor] = F.binary_cross_entropy_with_logits
        target_key: str = "label"
        kwargs: dict[str, Any] = field(default_factory=lambda: {"reduction": "none"})

    def __init__(self, config: Config) -> None:
        self.target_key = config.target_key
        self._fn = functools.partial(config.loss_fn, **config.kwargs)

    def __call__(self, prediction: Tensor, **batch: Any) -> LossOutput:
        if self.target_key not in batch:
            raise KeyError(f"Target key {self.target_key!r} not found in batch; keys: {list(batch)}")
        return {"loss": self._fn(prediction, batch[self.target_key])}


class TokenCrossEntropy:
    """Unreduced next-token CE over ``[B, S, V]`` logits, in fp32
    (``priml/baselines/nanochat/train_step.py:43-79``)."""

    class Config(Fig["TokenCrossEntropy"]):
        input_key: str = "tokens"
        target_key: str = "targets"
        ignore_index: int = -100
        softcap: float | None = None

    def __init__(self, config: Config | None = None) -> None:
        config = config or TokenCrossEntropy.Config()
        self.input_key = config.input_key
        self.target_key = config.target_key
        self.ignore_index = config.ignore_index
        self.softcap = config.softcap

    def __call__(self, prediction: Tensor, **batch: Any) -> LossOutput:
        return {"loss": ops.cross_entropy(prediction, batch[self.target_key], ignore_index=self.ignore_index,
                                          softcap=self.softcap)}  # fmt: skip

    def fused(self, model: Any, **batch: Any) -> LossOutput:
        """Loss straight from the model's hidden states (no logits tensor)."""
        return {"loss": model.token_loss(batch[self.input_key], batch[self.target_key], ignore_index=self.ignore_index)}


class WeightedSum:
    """``sum_i w_i * loss_i`` over member losses; member terms are reported under their names."""

    class Config(Fig["WeightedSum"]):
        losses: dict[str, Any] = field(default_factory=dict)
        weights: dict[str, float] = field(default_factory=dict)

    def __init__(self, config: Config) -> None:
        self.losses = {k: v.make() for k, v in config.losses.items()}
        self.weights = dict(config.weights)

    def __call__(self, prediction: Any, **batch: Any) -> LossOutput:
        out: LossOutput = {}
        total: Tensor | None = None
        for name, fn in self.losses.items():
            term = fn(prediction, **batch)["loss"]
            out[name] = term
            w = self.weights.get(name, 1.0)
            total = term * w if total is None else total + term * w
        assert total is not None
        out["loss"] = total
        return out


class AdversarialLoss:
    """Generator loss of a GAN step (``priml/loss/gan.py:19-90``), per sample:
    ``adversarial_weight * BCE(D(G(z)), 1) + content_weight * mean |G(z) - real|``."""

    class Config(Fig["AdversarialLoss"]):
        adversarial_weight: float = 1.0
        content_weight: float = 100.0

    def __init__(self, config: Config) -> None:
        self.adversarial_weight = config.adversarial_weight
        self.content_weight = config.content_weight

    def __call__(self, model_output: Tensor, *, fake_logits: Tensor, fake_media: Tensor, real_media: Tensor,
                 **batch: Any) -> LossOutput:  # fmt: skip
        del model_output, batch
        # BCE against "real" labels on logits is softplus(-logit)
        adversarial = F.softplus(-fake_logits.float()).flatten(1).mean(1)
        content = (fake_media.float() - real_media.float()).abs().flatten(1).mean(1)
        return {"loss": self.adversarial_weight * adversarial + self.content_weight * content}


_ = math


from priml_b200.loss.diffusion import DiffusionLoss  # noqa: E402
from priml_b200.loss.lpips import LPIPS, LPIPSLoss  # noqa: E402
from priml_b200.loss.policy_gradient import ClippedPolicyLoss, categorical_entropy, clipped_policy_loss  # noqa: E402
