"""Loads the in-tree CUDA extension ``priml_b200/ops/_C*.so``.

The extension is built ahead of time by ``priml_b200.ops.build`` (nvcc,
``-gencode arch=compute_100a,code=sm_100a``); it is never JIT-compiled at import
so that the exact binary that was built is the one that runs.
"""

from __future__ import annotations

import functools
import importlib
from types import ModuleType


@functools.cache
def _try_import() -> tuple[ModuleType | None, str]:
    try:
        import torch  # noqa: F401  -- libtorch must be loaded first

        mod = importlib.import_module("priml_b200.ops._C")
        return mod, ""
    except ImportError as exc:  # pragma: no cover - depends on build state
        return None, str(exc)


def native_available() -> bool:
    return _try_import()[0] is not None


def native() -> ModuleType:
    """The compiled extension; raises if it was not built."""
    mod, err = _try_import()
    if mod is None:
        raise RuntimeError(
            "priml_b200 CUDA extension is not built (run `python -m priml_b200.ops.build`); "
            f"import error: {err}"
        )
    return mod
