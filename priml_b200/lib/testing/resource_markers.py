"""Resource markers for pytest: one marker per external resource a test needs
(``priml/lib/testing/resource_markers.py``).

A resource marker is ``<family>_<resource>`` -- ``gpu_torch_cuda``,
``compute_distributed``, ``bench_throughput``. Registering the hook
(``pytest_collection_modifyitems`` below, re-exported from a conftest) gives
every marked test:

* the broad selector marks its resource implies (``gpu_* -> cuda``,
  ``bench_* -> performance``, ``compute_* -> slow``, ...), so ``-m "not cuda"``
  keeps working as resources are added;
* a timeout (the longest of its markers': a resource's own or its family's), unless
  the test sets one;
* a skip under ``CI`` (without ``RUN_INTEGRATION``) when the resource is one CI
  does not have.

An unregistered marker with a resource family prefix fails collection, so a typo
cannot silently drop a test from its selection. Markers are registered the usual
way (``markers = gpu_torch_cuda: ...`` in the ini file);
:func:`registered_resource_markers` reads them back.
"""

from __future__ import annotations

import os
from collections.abc import Iterable, Iterator, Sequence
from dataclasses import dataclass
from typing import Protocol

import pytest

__all__ = [
    "FAMILIES",
    "RESOURCES",
    "Resource",
    "apply_resource_markers",
    "pytest_collection_modifyitems",
    "registered_resource_markers",
    "resource_marker_aliases",
    "resource_marker_family",
    "resource_marker_timeout",
]


class MarkedItem(Protocol):
    """What the hook needs from a collected test."""

    def iter_markers(self, name: str | None = ...) -> Iterator[pytest.Mark]: ...

    def get_closest_marker(self, name: str) -> pytest.Mark | None: ...

    def add_marker(self, marker: str | pytest.MarkDecorator, *, append: bool = ...) -> None: ...


FAMILIES: dict[str, int] = {"bench": 600, "cli": 120, "compute": 300, "gpu": 300, "network": 180}
"""Resource family -> default timeout in seconds."""


@dataclass(frozen=True)
class Resource:
    aliases: tuple[str, ...]
    timeout: int | None = None  # None: the family's
    ci_skip: bool = False


RESOURCES: dict[str, Resource] = {
    "bench_throughput": Resource(("performance",), ci_skip=True),
    "bench_wallclock": Resource(("performance",), ci_skip=True),
    "bench_memory": Resource(("performance",), ci_skip=True),
    "cli_git": Resource(("integration",)),
    "cli_python_subprocess": Resource(("integration",), timeout=300),
    "compute_distributed": Resource(("slow",)),
    "compute_large_fixture": Resource(("slow",), timeout=180),
    "compute_training": Resource(("slow",)),
    "compute_torch_compile": Resource(("slow",), timeout=900),
    "gpu_torch_cuda": Resource(("cuda",), ci_skip=True),
    "gpu_multi": Resource(("cuda",), timeout=600, ci_skip=True),
    "gpu_nccl": Resource(("cuda",), timeout=600, ci_skip=True),
    "network_huggingface": Resource(("integration",)),
    "network_wandb": Resource(("integration",)),
}
"""Known resource markers."""


def resource_marker_family(marker: str) -> str:
    family, sep, _ = marker.partition("_")
    if not sep or family not in FAMILIES:
        raise pytest.UsageError(f"{marker!r} is not a resource marker (<family>_<resource>, family in {sorted(FAMILIES)})")
    return family


def resource_marker_aliases(marker: str) -> tuple[str, ...]:
    if marker not in RESOURCES:
        raise pytest.UsageError(f"Unknown resource marker: {marker}")
    return RESOURCES[marker].aliases


def resource_marker_timeout(marker: str) -> int:
    res = RESOURCES.get(marker)
    if res is not None and res.timeout is not None:
        return res.timeout
    return FAMILIES[resource_marker_family(marker)]


def registered_resource_markers(config: pytest.Config) -> tuple[str, ...]:
    names = (line.partition(":")[0].strip() for line in config.getini("markers"))
    return tuple(n for n in names if n.partition("_")[0] in FAMILIES and "_" in n)


def _check_known(item: MarkedItem, known: set[str]) -> None:
    for mark in item.iter_markers():
        family, sep, _ = mark.name.partition("_")
        if sep and family in FAMILIES and mark.name not in known:
            raise pytest.UsageError(f"Unknown resource marker: {mark.name}")


def apply_resource_markers(items: Sequence[MarkedItem], *, resource_markers: Iterable[str]) -> None:
    """Add alias marks, a timeout and the CI skip to each item that carries resource markers."""
    known = set(resource_markers)
    in_ci = bool(os.environ.get("CI")) and not os.environ.get("RUN_INTEGRATION")
    for item in items:
        _check_known(item, known)
        used = [m for m in known if item.get_closest_marker(m) is not None]
        if not used:
            continue
        have = {m.name for m in item.iter_markers()}  # the hook may run once per conftest: add nothing twice
        for alias in sorted({a for m in used for a in resource_marker_aliases(m)} - have):
            item.add_marker(getattr(pytest.mark, alias))
        if "timeout" not in have:
            item.add_marker(pytest.mark.timeout(max(resource_marker_timeout(m) for m in used)))
        if in_ci and "skip" not in have:
            skipped = sorted(m for m in used if RESOURCES[m].ci_skip)
            if skipped:
                item.add_marker(pytest.mark.skip(reason=f"{skipped[0]} is not available in CI (RUN_INTEGRATION=1 runs it)"))


@pytest.hookimpl(tryfirst=True)
def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    apply_resource_markers(items, resource_markers=registered_resource_markers(config))
