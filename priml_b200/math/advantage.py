"""Return / advantage estimators for RL (``priml/math/advantage.py:17-140``).

Both estimators are backward linear recurrences over time,
``y_t = b_t + a_t * y_{t+1}``. Instead of a Python loop of T dependent steps
(T tiny kernel launches on a GPU) they are solved with a log-depth parallel
scan (Hillis-Steele doubling over the affine maps), i.e. ceil(log2 T)
vectorized steps over ``[T, envs]``.
"""

from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["explained_variance", "generalized_advantage", "q_lambda_targets", "reverse_linear_scan"]


def reverse_linear_scan(a: Tensor, b: Tensor) -> Tensor:
    """Solve ``y_t = b_t + a_t * y_{t+1}`` (``y_T = 0``) along dim 0 in log depth."""
    y = b.clone()
    coef = a.clone()
    T = y.shape[0]
    offset = 1
    while offset < T:
        # y_t <- y_t + coef_t * y_{t+offset}; coef_t <- coef_t * coef_{t+offset}
        shifted_y = torch.zeros_like(y)
        shifted_c = torch.zeros_like(coef)
        shifted_y[: T - offset] = y[offset:]
        shifted_c[: T - offset] = coef[offset:]
        y = y + coef * shifted_y
        coef = coef * shifted_c
        offset *= 2
    return y


def generalized_advantage(*, rewards: Tensor, values: Tensor, dones: Tensor, last_value: Tensor, discount: float,
                          trace_decay: float) -> tuple[Tensor, Tensor]:  # fmt: skip
    """GAE (Schulman et al. 2015): ``A_t = delta_t + gamma lambda (1 - d_t) A_{t+1}`` with
    ``delta_t = r_t + gamma (1 - d_t) V_{t+1} - V_t`` and ``V_T = last_value``.

    ``rewards / values / dones``: ``[time, envs]``; returns (advantages, advantages + values).
    """
    live = 1.0 - dones.to(values.dtype)
    next_values = torch.cat([values[1:], last_value.unsqueeze(0).to(values.dtype)], dim=0)
    delta = rewards.to(values.dtype) + discount * live * next_values - values
    adv = reverse_linear_scan(discount * trace_decay * live, delta)
    return adv, adv + values


def q_lambda_targets(*, rewards: Tensor, q_values: Tensor, dones: Tensor, discount: float,
                     trace_decay: float) -> Tensor:  # fmt: skip
    """Peng's Q(lambda) targets from a policy's own Q-values (Gallici et al. 2024, PQN).

    ``G_t = r_t + gamma (1 - d_t) [(1 - lambda) max_a Q_{t+1} + lambda G_{t+1}]`` with
    ``G_{T-1} = r_{T-1} + gamma (1 - d_{T-1}) max_a Q_T``; a terminal step's target is its reward.
    ``q_values``: ``[time + 1, envs, actions]``.
    """
    if rewards.shape[0] == 0:
        raise ValueError("Q(lambda) needs a non-empty sequence")
    if q_values.shape[0] != rewards.shape[0] + 1:
        raise ValueError("Q(lambda) needs exactly one more Q-value step than rewards")
    dtype = rewards.dtype if rewards.is_floating_point() else q_values.dtype
    live = 1.0 - dones.to(dtype)
    greedy = q_values.max(dim=-1).values.to(dtype)
    T = rewards.shape[0]
    # b_t = r_t + gamma live_t ((1 - lambda) g_{t+1}) for t < T-1, and r + gamma live g_T at t = T-1;
    # a_t = gamma lambda live_t for t < T-1, and 0 at the last step.
    mix = torch.full((T, 1), 1.0 - trace_decay, dtype=dtype, device=rewards.device)
    mix[-1] = 1.0
    mix = mix.view(T, *([1] * (rewards.ndim - 1)))
    b = rewards.to(dtype) + discount * live * mix * greedy[1:]
    a = discount * trace_decay * live
    a = torch.cat([a[:-1], torch.zeros_like(a[-1:])], dim=0)
    return reverse_linear_scan(a, b)


def explained_variance(predictions: Tensor, targets: Tensor) -> Tensor:
    """``1 - Var(targets - predictions) / Var(targets)``; 0 when the targets are constant."""
    var_t = targets.var(unbiased=False)
    ratio = (targets - predictions).var(unbiased=False) / torch.where(var_t > 0, var_t, 1.0)
    return torch.where(var_t > 0, 1.0 - ratio, torch.zeros_like(var_t))
