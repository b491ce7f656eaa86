"""Test fixtures (``priml/testing/fixtures.py:24-113``)."""

from __future__ import annotations

import gc
from collections.abc import Iterator
from contextlib import contextmanager

import torch

__all__ = ["cleanup_cuda", "get_device", "poison_free_pool", "torch_compiler_isolation"]


def get_device() -> torch.device:
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


@contextmanager
def cleanup_cuda() -> Iterator[None]:
    """Collect garbage and release cached CUDA blocks before and after the block."""

    def _clean() -> None:
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
            torch.cuda.empty_cache()

    _clean()
    try:
        yield
    finally:
        _clean()


@contextmanager
def torch_compiler_isolation() -> Iterator[None]:
    """Reset Dynamo's process-global caches after a block that used ``torch.compile``."""
    try:
        yield
    finally:
        import sys

        if "torch._dynamo" in sys.modules:
            torch._dynamo.reset()  # noqa: SLF001


def poison_free_pool(*, blocks: int = 32, device: torch.device | str | None = None) -> None:
    """Fill and free ``blocks`` allocations of assorted sizes with NaN so that a later
    ``torch.empty`` that the code under test forgets to initialize reads NaN, not
    plausible leftovers."""
    dev = torch.device(device) if device is not None else get_device()
    keep = []
    for i in range(blocks):
        n = 1 << (8 + i % 14)
        keep.append(torch.full((n,), float("nan"), device=dev))
    del keep
