"""Access to the unmodified reference package, for parity tests and the reference bench arm.

The reference (rekursiv-ai/priml) is kept as a plain copy of its package under
``baseline/_ref`` at the repository root: its ``pip install`` fails offline (the
build backend is not in the wheelhouse). Its config trees import ``configgle``,
a git-only dependency that cannot be installed offline either, so
:func:`load_reference` registers ``priml_b200.config`` under that name: a
pure-Python implementation of the same public surface (``Fig``, ``Makeable``,
``Makes``, ``PartialConfig``, ``InlineConfig``, ``MutableNamespace``,
``copy_tree``, ``apply_overrides``, ``resolve_config``) that imports no kernel
code, so every model, optimizer, loss and strategy of the reference runs its own
code.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

__all__ = ["REFERENCE_ROOT", "load_reference", "reference_available"]

REFERENCE_ROOT = Path(__file__).resolve().parents[2] / "baseline" / "_ref"


def reference_available() -> bool:
    return (REFERENCE_ROOT / "priml" / "__init__.py").is_file()


def load_reference() -> None:
    """Make ``import priml`` resolve to the reference copy (idempotent)."""
    if not reference_available():
        raise FileNotFoundError(f"the reference package is not present under {REFERENCE_ROOT}")
    if str(REFERENCE_ROOT) not in sys.path:
        sys.path.insert(0, str(REFERENCE_ROOT))
    if "configgle" in sys.modules:
        return
    import priml_b200.config as standin

    root = types.ModuleType("configgle")
    root.__dict__.update({name: getattr(standin, name) for name in standin.__all__})
    walk = types.ModuleType("configgle.walk")
    walk.copy_tree = standin.copy_tree  # type: ignore[attr-defined]
    launch = types.ModuleType("configgle.launch")
    launch.resolve_config = standin.resolve_config  # type: ignore[attr-defined]
    root.walk, root.launch = walk, launch  # type: ignore[attr-defined]
    sys.modules.update({"configgle": root, "configgle.walk": walk, "configgle.launch": launch})
