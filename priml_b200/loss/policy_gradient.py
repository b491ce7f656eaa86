"""PPO objective terms (``priml/loss/policy_gradient.py:27-125``).

``clipped_policy_loss`` returns the clipped surrogate, the clipped value
regression, the mean entropy and two trust-region diagnostics over one flat
batch. Advantages are standardised with the batch's own mean and population
standard deviation (plus the dtype's epsilon, so a constant vector stays finite)
before entering the surrogate. The KL estimate is ``E[(r - 1) - log r]``
(non-negative, low variance).
"""

from __future__ import annotations

from typing import NamedTuple

import torch
from torch import Tensor

__all__ = ["ClippedPolicyLoss", "categorical_entropy", "clipped_policy_loss"]


class ClippedPolicyLoss(NamedTuple):
    policy: Tensor
    """Clipped surrogate (to minimise)."""
    value: Tensor
    """Clipped value regression, 0.5 x mean of the larger squared error."""
    entropy: Tensor
    """Mean policy entropy."""
    approx_kl: Tensor
    """Estimated KL from the behaviour policy, in nats."""
    clip_fraction: Tensor
    """Share of samples whose probability ratio left ``[1 - eps, 1 + eps]``."""


def clipped_policy_loss(*, log_probs: Tensor, behavior_log_probs: Tensor, advantages: Tensor, values: Tensor,
                        behavior_values: Tensor, targets: Tensor, entropy: Tensor,
                        clip_epsilon: float) -> ClippedPolicyLoss:  # fmt: skip
    log_ratio = log_probs - behavior_log_probs
    ratio = log_ratio.exp()
    spread = advantages.std(unbiased=False) + torch.finfo(advantages.dtype).eps
    adv = (advantages - advantages.mean()) / spread
    lo, hi = 1.0 - clip_epsilon, 1.0 + clip_epsilon
    surrogate = torch.minimum(ratio * adv, ratio.clamp(lo, hi) * adv)
    v_clipped = behavior_values + (values - behavior_values).clamp(-clip_epsilon, clip_epsilon)
    value = 0.5 * torch.maximum((values - targets).square(), (v_clipped - targets).square()).mean()
    return ClippedPolicyLoss(
        policy=-surrogate.mean(),
        value=value,
        entropy=entropy.mean(),
        approx_kl=(ratio - 1.0 - log_ratio).mean(),
        clip_fraction=((ratio - 1.0).abs() > clip_epsilon).to(ratio.dtype).mean(),
    )


def categorical_entropy(log_probs: Tensor) -> Tensor:
    """Entropy over the last axis of normalised log-probabilities; masked actions (``-inf``) add 0."""
    terms = log_probs.exp() * log_probs
    return -torch.where(torch.isneginf(log_probs), torch.zeros_like(terms), terms).sum(-1)
