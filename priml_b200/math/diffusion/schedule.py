"""Noise schedules in log-SNR form (``priml/math/diffusion/schedule.py:38-520``).

``x_t = alpha x + sigma eps``, ``snr = alpha^2 / sigma^2``. Corruptions map
log-SNR to log-sigma: variance preserving (``alpha^2 + sigma^2 = 1``, Kingma et
al. 2021) and rectified flow (``alpha + sigma = 1``, Liu et al. 2022).
Time parameterizations map ``log t`` (t in (0, 1], t = 1 pure noise) to
log-SNR: logit (``sigma = t`` under rectified flow), log-tan ("cosine", Nichol &
Dhariwal 2021 with the shift of Hoogeboom et al. 2023) and truncated-normal
inverse CDF ("logistic normal", Esser et al. 2024). Everything is computed in
log space.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor
from priml_b200.math.numeric import log1mexp, log_arctan_exp, log_tan_exp, logsubexp
from priml_b200.math.probability import log_cdf_truncated_normal, quantile_truncated_normal

__all__ = [
    "compute_log_alpha",
    "input_conditioning_identity",
    "input_conditioning_rectified_flow",
    "log_sigma_from_log_snr_per_rectified_flow",
    "log_sigma_from_log_snr_per_variance_preserving",
    "log_snr_from_log_sigma_per_rectified_flow",
    "log_snr_from_log_sigma_per_variance_preserving",
    "log_snr_from_log_time_per_logit",
    "log_snr_from_log_time_per_logtan",
    "log_snr_from_log_time_per_truncnormicdf",
    "log_time_from_log_snr_per_logit",
    "log_time_from_log_snr_per_logtan",
    "log_time_from_log_snr_per_truncnormicdf",
]


def compute_log_alpha(log_snr: Tensor, log_sigma: Tensor) -> Tensor:
    """``log alpha = log_snr / 2 + log sigma``."""
    return 0.5 * log_snr + log_sigma


def log_sigma_from_log_snr_per_variance_preserving(log_snr: Tensorable) -> Tensor:
    """``sigma^2 = 1 / (1 + snr)``: ``log sigma = logsigmoid(-log_snr) / 2``."""
    return 0.5 * F.logsigmoid(-convert_to_tensor(log_snr))


def _one_of(sigma: Tensorable | None, log_sigma: Tensorable | None) -> Tensor:
    if (sigma is None) == (log_sigma is None):
        raise ValueError("pass exactly one of sigma and log_sigma")
    return torch.log(convert_to_tensor(sigma)) if log_sigma is None else convert_to_tensor(log_sigma)


def log_snr_from_log_sigma_per_variance_preserving(*, sigma: Tensorable | None = None,
                                                   log_sigma: Tensorable | None = None) -> Tensor:  # fmt: skip
    """``log_snr = -logit(sigma^2) = -2 log sigma + log(1 - sigma^2)``."""
    ls = _one_of(sigma, log_sigma)
    return -2.0 * ls + log1mexp(2.0 * ls)


def log_sigma_from_log_snr_per_rectified_flow(log_snr: Tensorable) -> Tensor:
    """``sigma = 1 / (1 + sqrt(snr))``: ``log sigma = logsigmoid(-log_snr / 2)``."""
    return F.logsigmoid(-0.5 * convert_to_tensor(log_snr))


def log_snr_from_log_sigma_per_rectified_flow(*, sigma: Tensorable | None = None,
                                              log_sigma: Tensorable | None = None) -> Tensor:  # fmt: skip
    """``log_snr = -2 logit(sigma)``."""
    ls = _one_of(sigma, log_sigma)
    return -2.0 * (ls - log1mexp(ls))


def log_snr_from_log_time_per_logit(log_t: Tensorable, *, low: Tensorable = -20, high: Tensorable = 20) -> Tensor:
    """``log_snr = -2 logit(t)`` (so that ``sigma = t`` under rectified flow), clamped."""
    log_t, low, high = convert_to_tensor(log_t, low, high)
    return torch.clamp(-2.0 * (log_t - log1mexp(log_t)), low, high)


def log_time_from_log_snr_per_logit(log_snr: Tensorable) -> Tensor:
    return F.logsigmoid(-0.5 * convert_to_tensor(log_snr))


def _logtan_ab(shift: Tensor, low: Tensor, high: Tensor) -> tuple[Tensor, Tensor]:
    # log_snr(t) = -2 log tan(a t + b) + shift with the endpoints mapped to [high, low]
    log_b = log_arctan_exp(-0.5 * (high - shift))
    log_a = logsubexp(log_arctan_exp(-0.5 * (low - shift)), log_b)
    return log_a, log_b


def log_snr_from_log_time_per_logtan(log_t: Tensorable, *, shift: Tensorable = 0, low: Tensorable = -20,
                                     high: Tensorable = 20) -> Tensor:  # fmt: skip
    log_t, shift, low, high = convert_to_tensor(log_t, shift, low, high)
    shift = torch.clamp(shift, low, high)
    log_a, log_b = _logtan_ab(shift, low, high)
    log_angle = torch.logaddexp(log_a + log_t, log_b)
    return torch.clamp(-2.0 * log_tan_exp(log_angle) + shift, low, high)


def log_time_from_log_snr_per_logtan(log_snr: Tensorable, *, shift: Tensorable = 0, low: Tensorable = -20,
                                     high: Tensorable = 20) -> Tensor:  # fmt: skip
    log_snr, shift, low, high = convert_to_tensor(log_snr, shift, low, high)
    shift = torch.clamp(shift, low, high)
    log_a, log_b = _logtan_ab(shift, low, high)
    log_angle = log_arctan_exp(-0.5 * (log_snr - shift))
    return logsubexp(log_angle, log_b) - log_a


def log_snr_from_log_time_per_truncnormicdf(log_t: Tensorable, *, shift: Tensorable = 0, low: Tensorable = -20,
                                            high: Tensorable = 20, scale: Tensorable = 2) -> Tensor:  # fmt: skip
    """Truncated-normal inverse CDF with the bounds swapped, so t = 0 -> high and t = 1 -> low."""
    log_t, shift, low, high, scale = convert_to_tensor(log_t, shift, low, high, scale)
    shift = torch.clamp(shift, low, high)
    out = quantile_truncated_normal(log_t.exp(), loc=shift, scale=scale, low=high, high=low)
    return torch.clamp(out, low, high)


def log_time_from_log_snr_per_truncnormicdf(log_snr: Tensorable, *, shift: Tensorable = 0, low: Tensorable = -20,
                                            high: Tensorable = 20, scale: Tensorable = 2) -> Tensor:  # fmt: skip
    log_snr, shift, low, high, scale = convert_to_tensor(log_snr, shift, low, high, scale)
    shift = torch.clamp(shift, low, high)
    return log_cdf_truncated_normal(log_snr, loc=shift, scale=scale, low=high, high=low)


def input_conditioning_rectified_flow(x: Tensorable, log_snr: Tensorable) -> Tensor:
    """``x / sqrt(alpha^2 + sigma^2)`` under rectified flow (unit-variance model input;
    Karras et al. 2022's c_in with sigma_data = 1)."""
    x, log_snr = convert_to_tensor(x, log_snr)
    log_sigma = log_sigma_from_log_snr_per_rectified_flow(log_snr)
    log_alpha = compute_log_alpha(log_snr, log_sigma)
    return x * torch.exp(-0.5 * torch.logaddexp(2.0 * log_alpha, 2.0 * log_sigma))


def input_conditioning_identity(x: Tensorable, log_snr: Tensorable | None = None) -> Tensor:
    del log_snr
    return convert_to_tensor(x)
