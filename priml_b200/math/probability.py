"""Distribution functions and samplers (``priml/math/probability.py:22-660``).

Normal, uniform, logit-normal and truncated-normal densities / CDFs /
quantiles, the logit transform of an arbitrary base distribution, gamma /
chi-square / Student-t / categorical / logit-normal samplers and
log-gamma / log-beta helpers that stay accurate for large arguments
(Stirling series with its correction term).
"""

from __future__ import annotations

import math
from collections.abc import Callable

import torch
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor
from priml_b200.math.numeric import log1mexp

__all__ = [
    "cdf_logit_distribution",
    "cdf_logit_normal",
    "cdf_normal",
    "cdf_truncated_normal",
    "cdf_uniform",
    "lbeta",
    "log_cdf_truncated_normal",
    "log_gamma_correction",
    "log_gamma_difference",
    "ndtr",
    "ndtri",
    "pdf_logit_distribution",
    "pdf_logit_normal",
    "pdf_normal",
    "pdf_uniform",
    "quantile_logit_distribution",
    "quantile_logit_normal",
    "quantile_normal",
    "quantile_truncated_normal",
    "quantile_uniform",
    "random_categorical",
    "random_chi2",
    "random_gamma",
    "random_logit_normal",
    "random_student_t",
]

_LOG_SQRT_2PI = 0.5 * math.log(2.0 * math.pi)


def ndtr(x: Tensorable) -> Tensor:
    """Standard normal CDF ``0.5 erfc(-x / sqrt 2)``."""
    return torch.special.ndtr(convert_to_tensor(x))


def ndtri(p: Tensorable) -> Tensor:
    """Inverse of :func:`ndtr`."""
    return torch.special.ndtri(convert_to_tensor(p))


def pdf_normal(x: Tensorable, loc: Tensorable = 0.0, scale: Tensorable = 1.0) -> Tensor:
    x, loc, scale = convert_to_tensor(x, loc, scale)
    z = (x - loc) / scale
    return torch.exp(-0.5 * z * z - _LOG_SQRT_2PI) / scale


def cdf_normal(x: Tensorable, loc: Tensorable = 0.0, scale: Tensorable = 1.0) -> Tensor:
    x, loc, scale = convert_to_tensor(x, loc, scale)
    return torch.special.ndtr((x - loc) / scale)


def quantile_normal(p: Tensorable, *, loc: Tensorable = 0.0, scale: Tensorable = 1.0) -> Tensor:
    p, loc, scale = convert_to_tensor(p, loc, scale)
    return loc + scale * torch.special.ndtri(p)


def pdf_uniform(x: Tensorable, low: Tensorable = 0.0, high: Tensorable = 1.0) -> Tensor:
    x, low, high = convert_to_tensor(x, low, high)
    inside = (x >= low) & (x <= high)
    return torch.where(inside, 1.0 / (high - low), 0.0)


def cdf_uniform(x: Tensorable, low: Tensorable = 0.0, high: Tensorable = 1.0) -> Tensor:
    x, low, high = convert_to_tensor(x, low, high)
    return ((x - low) / (high - low)).clamp(0.0, 1.0)


def quantile_uniform(p: Tensorable, low: Tensorable = 0.0, high: Tensorable = 1.0) -> Tensor:
    p, low, high = convert_to_tensor(p, low, high)
    return low + p * (high - low)


def _logit(x: Tensor) -> Tensor:
    return torch.log(x) - torch.log1p(-x)


def pdf_logit_distribution(x: Tensorable, base_pdf: Callable[[Tensor], Tensor]) -> Tensor:
    """Density of ``Y = sigmoid(X)``: ``p_X(logit y) / (y (1 - y))``."""
    x = convert_to_tensor(x)
    return base_pdf(_logit(x)) / (x * (1.0 - x))


def cdf_logit_distribution(x: Tensorable, base_cdf: Callable[[Tensor], Tensor]) -> Tensor:
    return base_cdf(_logit(convert_to_tensor(x)))


def quantile_logit_distribution(x: Tensorable, base_quantile: Callable[[Tensor], Tensor]) -> Tensor:
    return torch.sigmoid(base_quantile(convert_to_tensor(x)))


def pdf_logit_normal(x: Tensorable, loc: Tensorable = 0.0, scale: Tensorable = 1.0) -> Tensor:
    return pdf_logit_distribution(x, lambda z: pdf_normal(z, loc, scale))


def cdf_logit_normal(x: Tensorable, loc: Tensorable = 0.0, scale: Tensorable = 1.0) -> Tensor:
    return cdf_logit_distribution(x, lambda z: cdf_normal(z, loc, scale))


def quantile_logit_normal(x: Tensorable, loc: Tensorable = 0.0, scale: Tensorable = 1.0) -> Tensor:
    return quantile_logit_distribution(x, lambda p: quantile_normal(p, loc=loc, scale=scale))


def _ndtr_diff(a: Tensor, b: Tensor) -> Tensor:
    """``Phi(b) - Phi(a)`` evaluated in whichever tail keeps precision (both upper: via -a, -b)."""
    upper = (a > 0) & (b > 0)
    return torch.where(upper, torch.special.ndtr(-a) - torch.special.ndtr(-b),
                       torch.special.ndtr(b) - torch.special.ndtr(a))  # fmt: skip


def _trunc_params(loc: Tensor, scale: Tensor, low: Tensor, high: Tensor) -> tuple[Tensor, Tensor]:
    return (low - loc) / scale, (high - loc) / scale


def cdf_truncated_normal(x: Tensorable, *, loc: Tensorable = 0.0, scale: Tensorable = 1.0,
                         low: Tensorable = -math.inf, high: Tensorable = math.inf) -> Tensor:  # fmt: skip
    """``(Phi(z) - Phi(alpha)) / (Phi(beta) - Phi(alpha))``; ``low > high`` gives the reversed
    (decreasing) map, which the schedules use."""
    x, loc, scale, low, high = convert_to_tensor(x, loc, scale, low, high)
    alpha, beta = _trunc_params(loc, scale, low, high)
    z = (x - loc) / scale
    return (_ndtr_diff(alpha, z) / _ndtr_diff(alpha, beta)).clamp(0.0, 1.0)


def log_cdf_truncated_normal(x: Tensorable, *, loc: Tensorable = 0.0, scale: Tensorable = 1.0,
                             low: Tensorable = -math.inf, high: Tensorable = math.inf) -> Tensor:  # fmt: skip
    """Log of :func:`cdf_truncated_normal`, from log-space tail probabilities so it stays
    finite far into either tail."""
    x, loc, scale, low, high = convert_to_tensor(x, loc, scale, low, high)
    alpha, beta = _trunc_params(loc, scale, low, high)
    z = (x - loc) / scale

    def log_abs_diff(a: Tensor, b: Tensor) -> Tensor:
        # log |Phi(b) - Phi(a)| using the tail (lower for negative, upper for positive args)
        use_upper = (a + b) > 0
        la = torch.where(use_upper, torch.special.log_ndtr(-a), torch.special.log_ndtr(a))
        lb = torch.where(use_upper, torch.special.log_ndtr(-b), torch.special.log_ndtr(b))
        hi, lo = torch.maximum(la, lb), torch.minimum(la, lb)
        return hi + log1mexp(torch.where(torch.isfinite(hi), lo - hi, -1.0))

    return log_abs_diff(alpha, z) - log_abs_diff(alpha, beta)


def quantile_truncated_normal(p: Tensorable, *, loc: Tensorable = 0.0, scale: Tensorable = 1.0,
                              low: Tensorable = -math.inf, high: Tensorable = math.inf) -> Tensor:  # fmt: skip
    """``loc + scale * Phi^-1(Phi(alpha) + p (Phi(beta) - Phi(alpha)))``, clamped to the bounds."""
    p, loc, scale, low, high = convert_to_tensor(p, loc, scale, low, high)
    alpha, beta = _trunc_params(loc, scale, low, high)
    # Work in whichever tail is accurate: the upper tail when the interval is on the right.
    upper = (alpha + beta) > 0
    pa = torch.where(upper, torch.special.ndtr(-alpha), torch.special.ndtr(alpha))
    pb = torch.where(upper, torch.special.ndtr(-beta), torch.special.ndtr(beta))
    u = pa + p * (pb - pa)
    z = torch.where(upper, -torch.special.ndtri(u), torch.special.ndtri(u))
    lo, hi = torch.minimum(low, high), torch.maximum(low, high)
    return torch.minimum(torch.maximum(loc + scale * z, lo), hi)


# ------------------------------------------------------------------ samplers
def _size(*samples_size: int) -> tuple[int, ...]:
    if len(samples_size) == 1 and isinstance(samples_size[0], (tuple, list, torch.Size)):
        return tuple(samples_size[0])
    return tuple(int(s) for s in samples_size)


def random_gamma(*samples_size: int, concentration: Tensorable, rate: Tensorable = 1.0,
                 dtype: torch.dtype | None = None, device: torch.device | None = None) -> Tensor:  # fmt: skip
    """``Gamma(concentration, rate)`` samples of shape ``(*samples_size, *params)``."""
    size = _size(*samples_size)
    c, r = convert_to_tensor(concentration, rate, dtype=dtype, device=device, dtype_hint=torch.float32)
    params = torch.broadcast_shapes(c.shape, r.shape)
    g = torch._standard_gamma(torch.broadcast_to(c, size + params).contiguous()).detach()  # noqa: SLF001
    return (g / r).clamp_min(torch.finfo(g.dtype).tiny)


def random_chi2(*samples_size: int, df: Tensorable, dtype: torch.dtype | None = None,
                device: torch.device | None = None) -> Tensor:  # fmt: skip
    d = convert_to_tensor(df, dtype=dtype, device=device, dtype_hint=torch.float32)
    return random_gamma(*samples_size, concentration=0.5 * d, rate=0.5)


def random_student_t(*samples_size: int, df: Tensorable, loc: Tensorable = 0.0, scale: Tensorable = 1.0,
                     dtype: torch.dtype | None = None, device: torch.device | None = None) -> Tensor:  # fmt: skip
    """``loc + scale * N / sqrt(Chi2(df) / df)``."""
    size = _size(*samples_size)
    df, loc, scale = convert_to_tensor(df, loc, scale, dtype=dtype, device=device, dtype_hint=torch.float32)
    params = torch.broadcast_shapes(df.shape, loc.shape, scale.shape)
    z = torch.randn(size + params, dtype=df.dtype, device=df.device)
    half = 0.5 * torch.broadcast_to(df, params)
    g = random_gamma(*size, concentration=half, rate=half)
    return loc + scale * z * torch.rsqrt(g)


def random_categorical(*samples_size: int, probs: Tensorable | None = None, logits: Tensorable | None = None,
                       dtype: torch.dtype | None = None, device: torch.device | None = None) -> Tensor:  # fmt: skip
    """Class indices of shape ``(*samples_size, *batch)`` by the Gumbel-max trick."""
    if (probs is None) == (logits is None):
        raise ValueError("pass exactly one of probs or logits")
    size = _size(*samples_size)
    lg = (torch.log(convert_to_tensor(probs, device=device, dtype_hint=torch.float32)) if logits is None
          else convert_to_tensor(logits, device=device, dtype_hint=torch.float32))  # fmt: skip
    u = torch.rand(size + lg.shape, dtype=lg.dtype if lg.is_floating_point() else torch.float32, device=lg.device)
    gumbel = -torch.log(-torch.log(u.clamp(torch.finfo(u.dtype).tiny, 1.0)))
    return (lg + gumbel).argmax(dim=-1).to(dtype or torch.int64)


def random_logit_normal(*samples_size: int, loc: Tensorable = 0.0, scale: Tensorable = 1.0,
                        dtype: torch.dtype | None = None, device: torch.device | None = None) -> Tensor:  # fmt: skip
    size = _size(*samples_size)
    loc, scale = convert_to_tensor(loc, scale, dtype=dtype, device=device, dtype_hint=torch.float32)
    params = torch.broadcast_shapes(loc.shape, scale.shape)
    return torch.sigmoid(loc + scale * torch.randn(size + params, dtype=loc.dtype, device=loc.device))


# ------------------------------------------------------------------ log-gamma / log-beta
def log_gamma_correction(x: Tensorable) -> Tensor:
    """``lgamma(x) - [(x - 1/2) log x - x + log sqrt(2 pi)]`` for ``x >= 8`` from the
    Stirling series ``sum_k B_2k / (2k (2k - 1) x^(2k-1))`` (first five terms)."""
    x = convert_to_tensor(x)
    inv = 1.0 / x
    inv2 = inv * inv
    # B2/2 = 1/12, B4/12 = -1/360, B6/30 = 1/1260, B8/56 = -1/1680, B10/90 = 1/1188
    series = 1.0 / 12 + inv2 * (-1.0 / 360 + inv2 * (1.0 / 1260 + inv2 * (-1.0 / 1680 + inv2 * (1.0 / 1188))))
    return series * inv


def _stirling(x: Tensor) -> Tensor:
    return (x - 0.5) * torch.log(x) - x + _LOG_SQRT_2PI + log_gamma_correction(x)


def log_gamma_difference(x: Tensorable, y: Tensorable) -> Tensor:
    """``lgamma(y) - lgamma(x + y)`` for ``y >= 8`` (and ``x >= 0``) without cancellation:
    ``-(y - 1/2) log1p(x/y) - x log(x + y) + x + c(y) - c(x + y)``."""
    x, y = convert_to_tensor(x, y)
    s = x + y
    return (-(y - 0.5) * torch.log1p(x / y) - x * torch.log(s) + x + log_gamma_correction(y)
            - log_gamma_correction(s))  # fmt: skip


def lbeta(x: Tensorable, y: Tensorable) -> Tensor:
    """``log B(x, y) = lgamma(x) + lgamma(y) - lgamma(x + y)``, with the large-argument
    cases done through the Stirling corrections."""
    x, y = convert_to_tensor(x, y)
    a, b = torch.minimum(x, y), torch.maximum(x, y)
    s = a + b
    both_big = a >= 8
    one_big = (b >= 8) & ~both_big
    a_big = torch.where(both_big, a, 8.0)
    b_big = torch.where(both_big | one_big, b, 8.0)
    s_big = a_big + b_big
    big = ((a_big - 0.5) * torch.log(a_big / s_big) + b_big * torch.log1p(-a_big / s_big) - 0.5 * torch.log(b_big)
           + _LOG_SQRT_2PI + log_gamma_correction(a_big) + log_gamma_correction(b_big) - log_gamma_correction(s_big))  # fmt: skip
    mixed = torch.lgamma(a) + log_gamma_difference(a, b_big)
    small = torch.lgamma(a) + torch.lgamma(b) - torch.lgamma(s)
    return torch.where(both_big, big, torch.where(one_big, mixed, small))
