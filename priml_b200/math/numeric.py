"""Numeric kernels used by the optimizers and losses (``priml/math/numeric.py``)."""

from __future__ import annotations

import math

import torch
from torch import Tensor

__all__ = [
    "kahan_sum",
    "log1mexp",
    "matrix_signum_via_newtonschulz",
    "polar_express",
    "safe_div",
    "safe_log",
    "safe_sqrt",
    "straight_through",
]

POLAR_EXPRESS_COEFFICIENTS: tuple[tuple[float, float, float], ...] = (
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
)
"""Five-step Polar-Express schedule (Amsel et al. 2025, arXiv:2505.16932)."""


def matrix_signum_via_newtonschulz(
    x: Tensor,
    coefficients: tuple[float, float, float] = (3.4445, -4.7750, 2.0315),
    steps: int = 5,
    eps: float = 1e-7,
) -> Tensor:
    """Quintic Newton-Schulz iteration toward ``U V^T`` of ``x = U S V^T``
    (Bernstein & Wan 2024; K. Jordan's Muon). ``x`` is ``[batch, rows, cols]``;
    runs in bf16 on the wide orientation, returns ``x``'s dtype."""
    a, b, c = coefficients
    dtype = x.dtype
    y = x.bfloat16()
    y = y / y.norm(dim=(-2, -1), keepdim=True).clamp(min=eps)
    tall = y.shape[-2] > y.shape[-1]
    if tall:
        y = y.transpose(-2, -1)
    for _ in range(steps):
        gram = y @ y.transpose(-1, -2)
        corr = torch.baddbmm(gram, gram, gram, beta=b, alpha=c)
        y = torch.baddbmm(y, corr, y, beta=a, alpha=1)
    if tall:
        y = y.transpose(-1, -2)
    return y.to(dtype)


def polar_express(x: Tensor, steps: int = 5, coefficients=POLAR_EXPRESS_COEFFICIENTS) -> Tensor:  # noqa: ANN001
    """Polar-Express orthogonalization in bf16 (norm scaled by 1.02 for safety)."""
    y = x.bfloat16()
    y = y / (y.norm(dim=(-2, -1), keepdim=True) * 1.02 + 1e-6)
    tall = y.size(-2) > y.size(-1)
    for a, b, c in coefficients[:steps]:
        if tall:
            gram = y.mT @ y
            y = a * y + y @ (b * gram + c * (gram @ gram))
        else:
            gram = y @ y.mT
            y = a * y + (b * gram + c * (gram @ gram)) @ y
    return y


def log1mexp(x: Tensor) -> Tensor:
    """``log(1 - exp(x))`` for ``x <= 0`` (Maechler 2012 split at ``-log 2``)."""
    return torch.where(x > -math.log(2.0), torch.log(-torch.expm1(x)), torch.log1p(-torch.exp(x)))


def kahan_sum(x: Tensor, dim: int = -1) -> Tensor:
    """Compensated summation along ``dim``."""
    x = x.movedim(dim, 0)
    s = torch.zeros_like(x[0])
    c = torch.zeros_like(x[0])
    for v in x:
        y = v - c
        t = s + y
        c = (t - s) - y
        s = t
    return s


def safe_div(a: Tensor, b: Tensor, eps: float = 1e-12) -> Tensor:
    return a / torch.where(b.abs() < eps, torch.full_like(b, eps).copysign(b), b)


def safe_log(x: Tensor, eps: float = 1e-12) -> Tensor:
    return torch.log(x.clamp_min(eps))


def safe_sqrt(x: Tensor, eps: float = 0.0) -> Tensor:
    return torch.sqrt(x.clamp_min(eps))


def straight_through(forward: Tensor, backward: Tensor) -> Tensor:
    """Value of ``forward`` with the gradient of ``backward``."""
    return backward + (forward - backward).detach()
