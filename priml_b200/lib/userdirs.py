"""Per-user base directories after the XDG Base Directory Specification (``priml/lib/userdirs.py``).

Each function returns a base directory; callers join their own namespace
(``cache_dir() / "priml_b200" / "kernels"``). Nothing is created.

==========  ===============  ==============  =============================
function    variable         Linux / BSD     macOS
==========  ===============  ==============  =============================
data_dir    XDG_DATA_HOME    ~/.local/share  ~/Library/Application Support
config_dir  XDG_CONFIG_HOME  ~/.config       ~/Library/Application Support
cache_dir   XDG_CACHE_HOME   ~/.cache        ~/Library/Caches
state_dir   XDG_STATE_HOME   ~/.local/state  ~/Library/Application Support
==========  ===============  ==============  =============================

An unset or empty variable means the platform default. On Windows every
function returns ``LOCALAPPDATA`` (default ``~/AppData/Local``). Two choices
differ from the letter of the specification, on purpose: a relative
``XDG_*_HOME`` is used as given (sandboxes and tests point these at relative
scratch dirs, and falling back to ``$HOME`` would escape them), and the
variables are honoured on macOS too.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

__all__ = ["cache_dir", "config_dir", "data_dir", "state_dir"]

# function -> (variable, Linux default under $HOME, macOS default under $HOME)
_TABLE = {
    "data": ("XDG_DATA_HOME", (".local", "share"), ("Library", "Application Support")),
    "config": ("XDG_CONFIG_HOME", (".config",), ("Library", "Application Support")),
    "cache": ("XDG_CACHE_HOME", (".cache",), ("Library", "Caches")),
    "state": ("XDG_STATE_HOME", (".local", "state"), ("Library", "Application Support")),
}


def _base(kind: str, platform: str | None) -> Path:
    platform = platform or sys.platform  # read at call time, so tests can patch sys.platform
    if platform == "win32":
        return Path(os.environ.get("LOCALAPPDATA") or Path.home() / "AppData" / "Local")
    var, linux, mac = _TABLE[kind]
    value = os.environ.get(var)
    if value:
        return Path(value)
    return Path.home().joinpath(*(mac if platform == "darwin" else linux))


def data_dir(*, platform: str | None = None) -> Path:
    """Durable user data worth backing up (``XDG_DATA_HOME``)."""
    return _base("data", platform)


def config_dir(*, platform: str | None = None) -> Path:
    """Settings the user chose (``XDG_CONFIG_HOME``)."""
    return _base("config", platform)


def cache_dir(*, platform: str | None = None) -> Path:
    """Reconstructible data: downloads, build products, memoised results (``XDG_CACHE_HOME``)."""
    return _base("cache", platform)


def state_dir(*, platform: str | None = None) -> Path:
    """What the application wrote to resume its work: logs, history (``XDG_STATE_HOME``)."""
    return _base("state", platform)
