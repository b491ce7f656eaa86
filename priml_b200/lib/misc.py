"""JSON freeze/thaw and light schema validation, object-tree traversal, XDG
directories (``priml/lib/custom_json.py``, ``priml/lib/traverse.py``,
``priml/lib/userdirs.py``)."""

from __future__ import annotations

import os
from collections.abc import Callable, Iterator, Mapping, Sequence
from pathlib import Path
from types import MappingProxyType
from typing import Any

__all__ = [
    "bool_val",
    "dict_val",
    "float_val",
    "int_val",
    "json_freeze",
    "json_unfreeze",
    "traverse",
    "user_cache_dir",
    "user_data_dir",
    "validate_json_schema",
]


def json_freeze(obj: Any) -> Any:
    """Immutable view: mappings -> MappingProxyType, sequences -> tuples (recursive)."""
    if isinstance(obj, Mapping):
        return MappingProxyType({k: json_freeze(v) for k, v in obj.items()})
    if isinstance(obj, Sequence) and not isinstance(obj, (str, bytes)):
        return tuple(json_freeze(v) for v in obj)
    return obj


def json_unfreeze(obj: Any) -> Any:
    if isinstance(obj, Mapping):
        return {k: json_unfreeze(v) for k, v in obj.items()}
    if isinstance(obj, Sequence) and not isinstance(obj, (str, bytes)):
        return [json_unfreeze(v) for v in obj]
    return obj


_TYPES: dict[str, Callable[[Any], bool]] = {
    "object": lambda v: isinstance(v, Mapping),
    "array": lambda v: isinstance(v, Sequence) and not isinstance(v, (str, bytes)),
    "string": lambda v: isinstance(v, str),
    "integer": lambda v: isinstance(v, int) and not isinstance(v, bool),
    "number": lambda v: isinstance(v, (int, float)) and not isinstance(v, bool),
    "boolean": lambda v: isinstance(v, bool),
    "null": lambda v: v is None,
}


def validate_json_schema(schema: Any, value: Any, path: str = "$") -> list[str]:
    """Errors of ``value`` against a JSON-schema subset (type, enum, min/max, properties, required, items)."""
    errs: list[str] = []
    if not isinstance(schema, Mapping):
        return errs
    t = schema.get("type")
    if t is not None:
        types = [t] if isinstance(t, str) else list(t)
        if not any(_TYPES.get(x, lambda v: True)(value) for x in types):
            return [f"{path}: expected {t}, got {type(value).__name__}"]
    if "enum" in schema and value not in schema["enum"]:
        errs.append(f"{path}: {value!r} not in {list(schema['enum'])}")
    if isinstance(value, (int, float)) and not isinstance(value, bool):
        if "minimum" in schema and value < schema["minimum"]:
            errs.append(f"{path}: {value} < minimum {schema['minimum']}")
        if "maximum" in schema and value > schema["maximum"]:
            errs.append(f"{path}: {value} > maximum {schema['maximum']}")
    if isinstance(value, Mapping):
        for req in schema.get("required", []):
            if req not in value:
                errs.append(f"{path}.{req}: required")
        for k, sub in schema.get("properties", {}).items():
            if k in value:
                errs += validate_json_schema(sub, value[k], f"{path}.{k}")
    if isinstance(value, Sequence) and not isinstance(value, (str, bytes)) and "items" in schema:
        for i, v in enumerate(value):
            errs += validate_json_schema(schema["items"], v, f"{path}[{i}]")
    return errs


def bool_val(value: Any, default: bool = False) -> bool:
    if isinstance(value, bool):
        return value
    if isinstance(value, str):
        return value.strip().lower() in ("1", "true", "yes", "on")
    return default if value is None else bool(value)


def float_val(value: Any, default: float = 0.0) -> float:
    try:
        return float(value)
    except (TypeError, ValueError):
        return default


def int_val(value: Any, default: int) -> int:
    try:
        return int(value)
    except (TypeError, ValueError):
        return default


def dict_val(value: Any) -> dict[str, Any]:
    return dict(value) if isinstance(value, Mapping) else {}


def traverse(obj: Any, visit: Callable[[str, Any], None] | None = None, path: str = "") -> Iterator[tuple[str, Any]]:
    """Depth-first (path, leaf) pairs over nested mappings / sequences / dataclass-like objects."""
    if isinstance(obj, Mapping):
        items = list(obj.items())
    elif isinstance(obj, Sequence) and not isinstance(obj, (str, bytes)):
        items = list(enumerate(obj))
    elif hasattr(obj, "__dataclass_fields__"):
        items = [(k, getattr(obj, k)) for k in obj.__dataclass_fields__]
    else:
        if visit is not None:
            visit(path, obj)
        yield path, obj
        return
    for k, v in items:
        yield from traverse(v, visit, f"{path}.{k}" if path else str(k))


def _xdg(env: str, fallback: str) -> Path:
    base = os.environ.get(env) or str(Path.home() / fallback)
    return Path(base) / "priml_b200"


def user_cache_dir() -> Path:
    return _xdg("XDG_CACHE_HOME", ".cache")


def user_data_dir() -> Path:
    return _xdg("XDG_DATA_HOME", ".local/share")
