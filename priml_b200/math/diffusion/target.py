"""Prediction targets (``priml/math/diffusion/target.py:56-440``).

For ``x_t = alpha x + sigma eps`` each parameterization returns what the
loss compares (``target`` vs ``predict``) and the model's implied clean
signal and noise (``x_clean`` / ``eps_clean``) for sampling:

* ``target_x`` / ``target_eps``: the model predicts x / eps;
* ``target_v``: ``v = alpha eps - sigma x`` (Salimans & Ho 2022), inverted as
  ``x = (alpha x_t - sigma v) / (alpha^2 + sigma^2)``,
  ``eps = (sigma x_t + alpha v) / (alpha^2 + sigma^2)``;
* ``target_rectified_flow``: ``v = eps - x`` (Liu et al. 2022), inverted as
  ``x = (x_t - sigma v) / (alpha + sigma)``, ``eps = (x_t + alpha v) / (alpha + sigma)``;
* ``target_v_x`` / ``target_v_eps``: v-parameterized model, loss in x / eps space.
"""

from __future__ import annotations

from typing import NamedTuple, Protocol

import torch
from torch import Tensor

from priml_b200.math.diffusion.schedule import compute_log_alpha

__all__ = ["TargetFn", "TargetResult", "target_eps", "target_rectified_flow", "target_v", "target_v_eps",
           "target_v_x", "target_x"]  # fmt: skip


class TargetResult(NamedTuple):
    target: Tensor | None
    predict: Tensor | None
    x_clean: Tensor
    eps_clean: Tensor


class TargetFn(Protocol):
    def __call__(self, model: Tensor, x_noisy: Tensor, log_snr: Tensor, log_sigma: Tensor, *,
                 x_original: Tensor | None = None, eps_original: Tensor | None = None) -> TargetResult: ...  # fmt: skip


def _coefs(log_snr: Tensor, log_sigma: Tensor) -> tuple[Tensor, Tensor]:
    return torch.exp(compute_log_alpha(log_snr, log_sigma)), torch.exp(log_sigma)


def target_x(model: Tensor, x_noisy: Tensor, log_snr: Tensor, log_sigma: Tensor, *,
             x_original: Tensor | None = None, eps_original: Tensor | None = None) -> TargetResult:  # fmt: skip
    del eps_original
    a, s = _coefs(log_snr, log_sigma)
    return TargetResult(x_original, model, model, (x_noisy - a * model) / s)


def target_eps(model: Tensor, x_noisy: Tensor, log_snr: Tensor, log_sigma: Tensor, *,
               x_original: Tensor | None = None, eps_original: Tensor | None = None) -> TargetResult:  # fmt: skip
    del x_original
    a, s = _coefs(log_snr, log_sigma)
    return TargetResult(eps_original, model, (x_noisy - s * model) / a, model)


def _from_v(v: Tensor, x_noisy: Tensor, a: Tensor, s: Tensor) -> tuple[Tensor, Tensor]:
    norm = a * a + s * s
    return (a * x_noisy - s * v) / norm, (s * x_noisy + a * v) / norm


def target_v(model: Tensor, x_noisy: Tensor, log_snr: Tensor, log_sigma: Tensor, *,
             x_original: Tensor | None = None, eps_original: Tensor | None = None) -> TargetResult:  # fmt: skip
    a, s = _coefs(log_snr, log_sigma)
    target = None if x_original is None or eps_original is None else a * eps_original - s * x_original
    x, e = _from_v(model, x_noisy, a, s)
    return TargetResult(target, model, x, e)


def target_rectified_flow(model: Tensor, x_noisy: Tensor, log_snr: Tensor, log_sigma: Tensor, *,
                          x_original: Tensor | None = None, eps_original: Tensor | None = None) -> TargetResult:  # fmt: skip
    a, s = _coefs(log_snr, log_sigma)
    target = None if x_original is None or eps_original is None else eps_original - x_original
    total = a + s
    return TargetResult(target, model, (x_noisy - s * model) / total, (x_noisy + a * model) / total)


def target_v_x(model: Tensor, x_noisy: Tensor, log_snr: Tensor, log_sigma: Tensor, *,
               x_original: Tensor | None = None, eps_original: Tensor | None = None) -> TargetResult:  # fmt: skip
    del eps_original
    a, s = _coefs(log_snr, log_sigma)
    x, e = _from_v(model, x_noisy, a, s)
    return TargetResult(x_original, x, x, e)


def target_v_eps(model: Tensor, x_noisy: Tensor, log_snr: Tensor, log_sigma: Tensor, *,
                 x_original: Tensor | None = None, eps_original: Tensor | None = None) -> TargetResult:  # fmt: skip
    del x_original
    a, s = _coefs(log_snr, log_sigma)
    x, e = _from_v(model, x_noisy, a, s)
    return TargetResult(eps_original, e, x, e)
