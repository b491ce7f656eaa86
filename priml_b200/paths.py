"""Working-directory resolution (``priml/paths.py:27-118``)."""

from __future__ import annotations

from pathlib import Path

__all__ = ["resolve_working_dir", "validated_output_path"]


def resolve_working_dir(working_dir: str | Path, base_dir: str | Path | None = None, **fmt: str) -> Path:
    """Format ``{placeholders}`` and anchor a relative path under ``base_dir``."""
    p = Path(str(working_dir).format(**fmt)) if fmt else Path(working_dir)
    if not p.is_absolute() and base_dir is not None:
        p = Path(base_dir) / p
    return p


def validated_output_path(path: str | Path, *, must_not_exist: bool = False, suffix: str | None = None) -> Path:
    p = Path(path)
    if suffix is not None and p.suffix != suffix:
        raise ValueError(f"{p} must end with {suffix}")
    if must_not_exist and p.exists():
        raise FileExistsError(p)
    p.parent.mkdir(parents=True, exist_ok=True)
    return p
