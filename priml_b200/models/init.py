"""Weight initializers with depth scaling (``priml/model/init.py:16-140``).

Every initializer divides by ``sqrt(depth + 1)`` when ``depth > 0``;
``call_init`` forwards only the keyword arguments an initializer accepts.
"""

from __future__ import annotations

import inspect
import math
from collections.abc import Callable

from torch import Tensor, nn

InitFn = Callable[[Tensor], object] | Callable[..., object]

__all__ = [
    "InitFn",
    "call_init",
    "dirac",
    "kaiming_normal",
    "kaiming_uniform",
    "mup_output",
    "normal",
    "truncated_normal",
    "unit_fan_in_uniform",
    "xavier_normal",
    "xavier_uniform",
    "zeros",
]


def call_init(fn: InitFn, t: Tensor, **kwargs: object) -> None:
    """Call ``fn(t, **kwargs)`` passing only keywords ``fn`` declares."""
    try:
        params = inspect.signature(fn).parameters
        if not any(p.kind is p.VAR_KEYWORD for p in params.values()):
            kwargs = {k: v for k, v in kwargs.items() if k in params and params[k].kind is p_kw}
    except (TypeError, ValueError):
        kwargs = {}
    fn(t, **kwargs)


p_kw = inspect.Parameter.KEYWORD_ONLY


def _depth_scale(w: Tensor, depth: int) -> None:
    if depth > 0:
        w.data.div_(math.sqrt(depth + 1))


def kaiming_uniform(w: Tensor, *, depth: int = 1) -> None:
    nn.init.kaiming_uniform_(w, a=math.sqrt(5))
    _depth_scale(w, depth)


def kaiming_normal(w: Tensor, *, depth: int = 1) -> None:
    nn.init.kaiming_normal_(w, a=math.sqrt(5))
    _depth_scale(w, depth)


def xavier_uniform(w: Tensor, *, depth: int = 1) -> None:
    nn.init.xavier_uniform_(w)
    _depth_scale(w, depth)


def xavier_normal(w: Tensor, *, depth: int = 1) -> None:
    nn.init.xavier_normal_(w)
    _depth_scale(w, depth)


def normal(w: Tensor, *, std: float = 0.02, depth: int = 1) -> None:
    nn.init.normal_(w, std=std)
    _depth_scale(w, depth)


def zeros(w: Tensor, *, depth: int = 1) -> None:
    del depth
    nn.init.zeros_(w)


def truncated_normal(
    w: Tensor,
    *,
    std: float = 0.02,
    depth: int = 1,
    lower: float = -2.0,
    upper: float = 2.0,
    variance_correction: bool = False,
) -> None:
    """Truncated normal on ``[lower*std, upper*std]``; with ``variance_correction``
    ``std`` is divided by the standard deviation of the unit normal truncated to
    ``[lower, upper]`` so the realized spread equals the request."""
    if variance_correction:
        if std == 0:
            nn.init.zeros_(w)
            return
        z = 0.5 * (math.erf(upper / math.sqrt(2)) - math.erf(lower / math.sqrt(2)))
        phi = lambda t: math.exp(-0.5 * t * t) / math.sqrt(2 * math.pi)  # noqa: E731
        var = 1.0 - (upper * phi(upper) - lower * phi(lower)) / z - ((phi(upper) - phi(lower)) / z) ** 2
        std = std / math.sqrt(var)
    nn.init.trunc_normal_(w, std=std, a=lower * std, b=upper * std)
    _depth_scale(w, depth)


def unit_fan_in_uniform(w: Tensor, *, depth: int = -1) -> None:
    """Uniform on ``±sqrt(3/fan_in)``; depth is ignored."""
    del depth
    bound = math.sqrt(3.0 / w.shape[-1])
    nn.init.uniform_(w, -bound, bound)


def mup_output(w: Tensor, *, depth: int = 1) -> None:
    fan_in = w.shape[1] if w.ndim >= 2 else w.shape[0]
    nn.init.normal_(w, std=1.0 / fan_in)
    _depth_scale(w, depth)


def dirac(w: Tensor) -> None:
    nn.init.dirac_(w)
