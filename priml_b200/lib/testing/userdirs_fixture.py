"""Autouse fixture that points every :mod:`priml_b200.lib.userdirs` lookup at a per-test directory.

Re-export it from a ``conftest.py``::

    from priml_b200.lib.testing.userdirs_fixture import isolate_user_dirs  # noqa: F401

A test that writes through ``cache_dir()`` and friends then writes under its own
``tmp_path`` rather than into the developer's real directories, and an
assertion can call the helper instead of spelling one platform's layout.
Module-level constants computed at import time are out of its reach.
"""

from __future__ import annotations

from collections.abc import Iterator
from pathlib import Path

import pytest

__all__ = ["isolate_user_dirs"]

_VARS = ("XDG_DATA_HOME", "XDG_CONFIG_HOME", "XDG_CACHE_HOME", "XDG_STATE_HOME", "LOCALAPPDATA")


@pytest.fixture(autouse=True)
def isolate_user_dirs(tmp_path: Path, monkeypatch: pytest.MonkeyPatch) -> Iterator[Path]:
    root = tmp_path / "userdirs"
    for var in _VARS:
        monkeypatch.setenv(var, str(root / var.lower()))
    yield root
