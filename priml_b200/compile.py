"""Compilation helpers (``priml/compile.py:26-131``).

The hot paths here are hand-written kernels run eagerly; these helpers remain
for user code that wants ``torch.compile`` on its own functions, compiled lazily
on first call so importing a module never pays for it.
"""

from __future__ import annotations

import functools
from collections.abc import Callable
from typing import Any

import torch

__all__ = ["lazy_assume_constant_result", "lazy_torch_compile", "trace_compile"]


def lazy_torch_compile(*compile_args: Any, **compile_kwargs: Any) -> Callable[..., Any]:
    def deco(fn: Callable[..., Any]) -> Callable[..., Any]:
        compiled: list[Callable[..., Any]] = []

        @functools.wraps(fn)
        def wrapper(*args: Any, **kwargs: Any) -> Any:
            if not compiled:
                compiled.append(torch.compile(fn, *compile_args, **compile_kwargs))
            return compiled[0](*args, **kwargs)

        return wrapper

    return deco


def lazy_assume_constant_result(fn: Callable[..., Any]) -> Callable[..., Any]:
    cache: dict[Any, Any] = {}

    @functools.wraps(fn)
    def wrapper(*args: Any) -> Any:
        if args not in cache:
            cache[args] = fn(*args)
        return cache[args]

    return wrapper


def trace_compile(fn: Callable[..., Any], *example: Any) -> Any:
    """``torch.jit.trace`` a function on example inputs."""
    return torch.jit.trace(fn, example)
