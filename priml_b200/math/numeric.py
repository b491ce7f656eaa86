"""Numeric kernels used by the optimizers and losses (``priml/math/numeric.py``)."""

from __future__ import annotations

import math

from collections.abc import Sequence

import torch
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor

__all__ = [
    "custom_grad",
    "kahan_sum",
    "log1mexp",
    "log1psquare",
    "log_arctan_exp",
    "log_cosh",
    "log_cumsum_exp",
    "log_modulus",
    "log_tan_exp",
    "logerfc",
    "logmeanexp",
    "logsubexp",
    "matrix_signum_via_newtonschulz",
    "mesh_arange",
    "polar_express",
    "power_transform",
    "power_transform_inverse",
    "safe_div",
    "safe_log",
    "safe_pow",
    "safe_rsqrt",
    "safe_sqrt",
    "safe_xlogy",
    "sinh_arcsinh",
    "sinh_arcsinh_inverse",
    "smootherstep",
    "smoothstep",
    "smoothstep_inverse",
    "soft_threshold",
    "softcap",
    "softmax_centered",
    "softmax_centered_inverse",
    "softplus_inverse",
    "softsign",
    "softsign_inverse",
    "sqrt1pm1",
    "ste_clamp",
    "ste_round",
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
    if y.is_cuda:
        from priml_b200.ops.orthogonalize import newton_schulz_steps

        return newton_schulz_steps(y, [(a, b, c)] * steps).to(dtype)
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
    if y.is_cuda:
        from priml_b200.ops.orthogonalize import newton_schulz_steps

        return newton_schulz_steps(y, coefficients[:steps])
    tall = y.size(-2) > y.size(-1)
    for a, b, c in coefficients[:steps]:
        if tall:
            gram = y.mT @ y
            y = a * y + y @ (b * gram + c * (gram @ gram))
        else:
            gram = y @ y.mT
            y = a * y + (b * gram + c * (gram @ gram)) @ y
    return y


# ------------------------------------------------------------------ log-space helpers
def log1mexp(x: Tensorable) -> Tensor:
    """``log(1 - exp(x))`` for ``x <= 0``, switching at ``-log 2`` between
    ``log(-expm1(x))`` and ``log1p(-exp(x))`` (Maechler 2012)."""
    x = convert_to_tensor(x)
    near_zero = x > -math.log(2.0)
    a = torch.where(near_zero, x, -1.0)
    b = torch.where(near_zero, -1.0, x)
    return torch.where(near_zero, torch.log(-torch.expm1(a)), torch.log1p(-torch.exp(b)))


def logsubexp(x: Tensorable, y: Tensorable, *, return_sign: bool = False) -> Tensor | tuple[Tensor, Tensor]:
    """``log|exp(x) - exp(y)|`` = ``max + log1mexp(min - max)``; with ``return_sign`` also
    ``sign(exp(x) - exp(y))``."""
    x, y = convert_to_tensor(x, y)
    hi, lo = torch.maximum(x, y), torch.minimum(x, y)
    diff = lo - hi
    finite = torch.isfinite(hi)
    out = torch.where(finite, hi + log1mexp(torch.where(finite, diff, -1.0)), hi)
    if return_sign:
        return out, torch.where(x >= y, 1.0, -1.0).to(out.dtype)
    return out


def log_arctan_exp(x: Tensorable) -> Tensor:
    """``log(arctan(exp(x)))``: ``x + log(arctan(u) / u)`` (u = e^x) below 0, the
    complement ``log(pi/2 - arctan(e^-x))`` above."""
    x = convert_to_tensor(x)
    neg = x <= 0
    u = torch.exp(torch.where(neg, x, 0.0))
    ratio = torch.where(u > 1e-4, torch.arctan(u) / torch.where(u > 1e-4, u, 1.0), 1.0 - u * u / 3.0)
    small = x + torch.log(ratio)
    large = torch.log(math.pi / 2 - torch.arctan(torch.exp(-torch.where(neg, 1.0, x))))
    return torch.where(neg, small, large)


def log_tan_exp(x: Tensorable) -> Tensor:
    """``log(tan(exp(x)))`` for ``x < log(pi/2)``: ``x + log(tan(u) / u)`` keeps small
    angles exact."""
    x = convert_to_tensor(x)
    u = torch.exp(x)
    ratio = torch.where(u > 1e-4, torch.tan(u) / torch.where(u > 1e-4, u, 1.0), 1.0 + u * u / 3.0)
    return x + torch.log(ratio)


def logerfc(x: Tensorable) -> Tensor:
    """``log(erfc(x))``; for ``x >= 0`` through ``log(erfcx(x)) - x^2`` (no underflow)."""
    x = convert_to_tensor(x)
    pos = x >= 0
    xp = torch.where(pos, x, 0.0)
    xn = torch.where(pos, -1.0, x)
    return torch.where(pos, torch.log(torch.special.erfcx(xp)) - xp * xp, torch.log(torch.erfc(xn)))


def log_cosh(x: Tensorable) -> Tensor:
    """``log(cosh(x)) = |x| + log1p(exp(-2|x|)) - log 2``."""
    x = convert_to_tensor(x)
    a = x.abs()
    return a + torch.log1p(torch.exp(-2.0 * a)) - math.log(2.0)


def softplus_inverse(x: Tensorable) -> Tensor:
    """Inverse of softplus: ``x + log(-expm1(-x))`` for ``x > 0``."""
    x = convert_to_tensor(x)
    return x + torch.log(-torch.expm1(-x))


def log1psquare(x: Tensorable) -> Tensor:
    """``log(1 + x^2)``, as ``2 log|x| + log1p(1/x^2)`` for ``|x| > 1``."""
    x = convert_to_tensor(x)
    a = x.abs()
    big = a > 1.0
    ab = torch.where(big, a, 2.0)
    return torch.where(big, 2.0 * torch.log(ab) + torch.log1p(1.0 / (ab * ab)), torch.log1p(x * x))


def logmeanexp(x: Tensorable, dim: int | Sequence[int] = -1, keepdim: bool = False) -> Tensor:
    x = convert_to_tensor(x)
    dims = (dim,) if isinstance(dim, int) else tuple(dim)
    n = math.prod(x.shape[d] for d in dims)
    return torch.logsumexp(x, dim=dims, keepdim=keepdim) - math.log(n)


def log_cumsum_exp(x: Tensorable, dim: int = -1) -> Tensor:
    return torch.logcumsumexp(convert_to_tensor(x), dim=dim)


# ------------------------------------------------------------------ grids and sums
def mesh_arange(end: Sequence[int] | int, *, start: Sequence[int] | int = 0, step: Sequence[int] | int = 1,
                dtype: torch.dtype = torch.long, device: torch.device | str | None = None) -> Tensor:  # fmt: skip
    """All integer grid points ``start <= p < end`` (row-major), shape ``[count, ndim]``."""
    from priml_b200.math.basic import broadcast_sequences

    starts, ends, steps = broadcast_sequences(start, end, step)
    axes = [torch.arange(a, b, c, dtype=dtype, device=device) for a, b, c in zip(starts, ends, steps, strict=True)]
    return torch.stack(torch.meshgrid(*axes, indexing="ij"), dim=-1).reshape(-1, len(axes))


def kahan_sum(x: Tensorable, dim: int | None = None, keepdim: bool = False) -> Tensor:
    """Compensated (Neumaier) summation along ``dim`` (all elements when None): the
    running compensation collects the low-order bits each addition drops, taking
    the error from whichever operand is smaller in magnitude."""
    x = convert_to_tensor(x)
    ndim = x.ndim
    if dim is None:
        v = x.reshape(-1, *([1] * 0))
        axis = 0
    else:
        v = x
        axis = dim % max(ndim, 1)
    v = v.movedim(axis, 0)
    total = torch.zeros_like(v[0]) if v.shape[0] else v.new_zeros(v.shape[1:])
    comp = torch.zeros_like(total)
    for term in v:
        s = total + term
        comp = comp + torch.where(total.abs() >= term.abs(), (total - s) + term, (term - s) + total)
        total = s
    out = total + comp
    if keepdim:
        if dim is None:
            out = out.reshape([1] * ndim)
        else:
            out = out.unsqueeze(axis)
    return out


# ------------------------------------------------------------------ smooth maps
def softcap(x: Tensorable, cap: Tensorable = 1.0) -> Tensor:
    """``cap * tanh(x / cap)`` computed in fp32, returned in the input dtype."""
    dtype = torch.as_tensor(x).dtype
    x, cap = convert_to_tensor(x, cap, dtype=torch.float32)
    return (cap * torch.tanh(x / cap)).to(dtype)


def smoothstep(x: Tensorable) -> Tensor:
    """``3x^2 - 2x^3`` on ``[0, 1]`` (clamped outside)."""
    x = convert_to_tensor(x).clamp(0.0, 1.0)
    return x * x * (3.0 - 2.0 * x)


def smoothstep_inverse(y: Tensorable) -> Tensor:
    """Inverse of :func:`smoothstep` in closed form: ``1/2 - sin(arcsin(1 - 2y) / 3)``."""
    y = convert_to_tensor(y).clamp(0.0, 1.0)
    return 0.5 - torch.sin(torch.arcsin(1.0 - 2.0 * y) / 3.0)


def smootherstep(x: Tensorable) -> Tensor:
    """Perlin's ``6x^5 - 15x^4 + 10x^3`` on ``[0, 1]`` (clamped outside)."""
    x = convert_to_tensor(x).clamp(0.0, 1.0)
    return x * x * x * (x * (6.0 * x - 15.0) + 10.0)


def soft_threshold(x: Tensorable, threshold: Tensorable) -> Tensor:
    """Proximal map of ``threshold * |x|``: ``sign(x) * max(|x| - threshold, 0)``."""
    x, threshold = convert_to_tensor(x, threshold)
    return torch.sign(x) * torch.relu(x.abs() - threshold)


def sqrt1pm1(x: Tensorable) -> Tensor:
    """``sqrt(1 + x) - 1`` without cancellation: ``x / (sqrt(1 + x) + 1)``."""
    x = convert_to_tensor(x)
    return x / (torch.sqrt(1.0 + x) + 1.0)


def log_modulus(x: Tensorable) -> Tensor:
    """John-Draper log-modulus ``sign(x) log1p(|x|)``."""
    x = convert_to_tensor(x)
    return torch.sign(x) * torch.log1p(x.abs())


def softsign(x: Tensorable) -> Tensor:
    x = convert_to_tensor(x)
    return x / (1.0 + x.abs())


def softsign_inverse(y: Tensorable) -> Tensor:
    y = convert_to_tensor(y)
    return y / (1.0 - y.abs())


def power_transform(x: Tensorable, power: float) -> Tensor:
    """``(1 + power x)^(1/power)`` (``exp(x)`` at power 0) -- the inverse Box-Cox map."""
    x = convert_to_tensor(x)
    if power == 0:
        return torch.exp(x)
    return safe_pow(1.0 + power * x, 1.0 / power)


def power_transform_inverse(y: Tensorable, power: float) -> Tensor:
    y = convert_to_tensor(y)
    if power == 0:
        return torch.log(y)
    return (torch.pow(y, power) - 1.0) / power


def softmax_centered(x: Tensorable, dim: int = -1) -> Tensor:
    """Softmax over ``x`` with an extra zero logit appended: R^n -> interior of the n-simplex."""
    x = convert_to_tensor(x)
    pivot = torch.zeros_like(x.narrow(dim, 0, 1))
    return torch.softmax(torch.cat([x, pivot], dim=dim), dim=dim)


def softmax_centered_inverse(y: Tensorable, dim: int = -1) -> Tensor:
    y = convert_to_tensor(y)
    logs = torch.log(y)
    n = y.shape[dim]
    return logs.narrow(dim, 0, n - 1) - logs.narrow(dim, n - 1, 1)


def sinh_arcsinh(x: Tensorable, skewness: Tensorable = 0.0, tailweight: Tensorable = 1.0) -> Tensor:
    """Jones-Pewsey sinh-arcsinh map ``sinh((asinh(x) + skewness) * tailweight)``."""
    x, skewness, tailweight = convert_to_tensor(x, skewness, tailweight)
    return torch.sinh((torch.asinh(x) + skewness) * tailweight)


def sinh_arcsinh_inverse(y: Tensorable, skewness: Tensorable = 0.0, tailweight: Tensorable = 1.0) -> Tensor:
    y, skewness, tailweight = convert_to_tensor(y, skewness, tailweight)
    return torch.sinh(torch.asinh(y) / tailweight - skewness)


# ------------------------------------------------------------------ gradient surgery
def custom_grad(*, actual: Tensor, phantom: Tensor) -> Tensor:
    """The value of ``actual`` with the gradient of ``phantom``."""
    return actual.detach() + (phantom - phantom.detach())


def straight_through(forward: Tensor, backward: Tensor) -> Tensor:
    """The value of ``forward`` with the gradient of ``backward``."""
    return custom_grad(actual=forward, phantom=backward)


def ste_round(x: Tensorable, scale: Tensorable = 1.0) -> Tensor:
    x, scale = convert_to_tensor(x, scale)
    return custom_grad(actual=torch.round(x * scale) / scale, phantom=x)


def ste_clamp(input: Tensorable, min: float | Tensor | None = None, max: float | Tensor | None = None) -> Tensor:  # noqa: A001, A002
    x = convert_to_tensor(input)
    return custom_grad(actual=torch.clamp(x, min, max), phantom=x)


# ------------------------------------------------------------------ safe elementary functions
# Each masks the argument before the unsafe op (so the discarded branch has a
# finite gradient) and then selects the convention value ("double where").
def safe_log(input: Tensorable) -> Tensor:  # noqa: A002
    """``log(x)`` for ``x > 0``, ``-inf`` otherwise, with finite gradients."""
    x = convert_to_tensor(input)
    ok = x > 0
    return torch.where(ok, torch.log(torch.where(ok, x, 1.0)), -math.inf)


def safe_xlogy(input: Tensorable, other: Tensorable) -> Tensor:  # noqa: A002
    """``x log(y)``, exactly 0 where ``x == 0`` (whatever ``y``)."""
    x, y = convert_to_tensor(input, other)
    return torch.xlogy(x, torch.where(x == 0, 1.0, y))


def safe_sqrt(input: Tensorable) -> Tensor:  # noqa: A002
    """``sqrt(x)`` for ``x > 0``, 0 otherwise, with finite gradients."""
    x = convert_to_tensor(input)
    ok = x > 0
    return torch.where(ok, torch.sqrt(torch.where(ok, x, 1.0)), 0.0)


def safe_rsqrt(input: Tensorable) -> Tensor:  # noqa: A002
    """``1/sqrt(x)``: ``+inf`` at 0 (the limit from above), 0 for negatives."""
    x = convert_to_tensor(input)
    ok = x > 0
    return torch.where(ok, torch.rsqrt(torch.where(ok, x, 1.0)), torch.where(x == 0, math.inf, 0.0))


def safe_pow(base: Tensorable, exponent: Tensorable) -> Tensor:
    """``base ** exponent`` for positive bases; ``0 ** 0 = 1`` and 0 for other non-positive bases."""
    b, e = convert_to_tensor(base, exponent)
    ok = b > 0
    return torch.where(ok, torch.pow(torch.where(ok, b, 1.0), e), torch.where((b == 0) & (e == 0), 1.0, 0.0))


def safe_div(a: Tensor, b: Tensor, eps: float = 1e-12) -> Tensor:
    """``a / b`` with ``|b|`` floored at ``eps`` (sign kept)."""
    return a / torch.where(b.abs() < eps, torch.full_like(b, eps).copysign(b), b)
