"""JSON helpers: frozen/thawed JSON values, a small schema checker, value coercion,
and a type-directed dataclass <-> JSON codec (``priml/lib/custom_json.py``).

The codec's wire format is the reference's, so documents written by either side
decode on the other:

* a dataclass encodes as an object of its ``init`` fields plus ``"__type__"``
  (the class name), which selects the member when a field's annotation is a
  union of dataclasses;
* ``bytes`` (base64), ``Path``, ``UUID``, ``datetime`` (ISO 8601) and ``Enum``
  (its value) encode as plain JSON values; where a union names two or more of
  them the value is wrapped as ``{"__scalar__": type name, "__value__": ...}``;
* sets encode as sorted lists, tuples and lists as lists, mappings as objects.

Decoding is driven by the target class's resolved annotations, coerces the
usual JSON looseness (``"3"`` to an int field, ``"false"`` to a bool), and
rejects keys that name no constructor parameter with :class:`SchemaError`.
"""

from __future__ import annotations

import base64
import types
from collections.abc import Callable, Mapping, Sequence
from collections.abc import Set as AbstractSet
from dataclasses import fields, is_dataclass
from datetime import datetime
from enum import Enum
from functools import cache
from pathlib import Path
from typing import Any, Final, TypeVar, Union, get_args, get_origin, get_type_hints
from uuid import UUID

__all__ = [
    "JsonCodec",
    "SchemaError",
    "bool_val",
    "dataclass_from_json",
    "dataclass_to_json",
    "datetime_val",
    "decode",
    "dict_val",
    "dicts_val",
    "float_val",
    "int_val",
    "json_freeze",
    "json_unfreeze",
    "list_val",
    "str_val",
    "validate_json_schema",
]

T = TypeVar("T")

TYPE_TAG: Final = "__type__"
SCALAR_TAG: Final = "__scalar__"
VALUE_TAG: Final = "__value__"


# ---------------------------------------------------------------------------- freeze / thaw
def json_freeze(obj: Any) -> Any:
    """Immutable copy: mappings become ``MappingProxyType``, sequences tuples."""
    if isinstance(obj, Mapping):
        return types.MappingProxyType({k: json_freeze(v) for k, v in obj.items()})
    if isinstance(obj, Sequence) and not isinstance(obj, str | bytes | bytearray):
        return tuple(json_freeze(v) for v in obj)
    return obj


def json_unfreeze(obj: Any) -> Any:
    """Plain ``dict`` / ``list`` copy of a (possibly frozen) JSON value; keys become strings."""
    if isinstance(obj, Mapping):
        return {str(k): json_unfreeze(v) for k, v in obj.items()}
    if isinstance(obj, tuple | list):
        return [json_unfreeze(v) for v in obj]
    return obj


# ---------------------------------------------------------------------------- schema subset
_TYPE_CHECKS: dict[str, Callable[[Any], bool]] = {
    "object": lambda v: isinstance(v, Mapping),
    "array": lambda v: isinstance(v, list),
    "string": lambda v: isinstance(v, str),
    "integer": lambda v: isinstance(v, int) and not isinstance(v, bool),
    "number": lambda v: isinstance(v, int | float) and not isinstance(v, bool),
    "boolean": lambda v: isinstance(v, bool),
    "null": lambda v: v is None,
}


def validate_json_schema(schema: Any, value: Any) -> list[str]:
    """Issues of ``value`` against a JSON Schema subset, as readable strings (empty when valid).

    Understood keywords: ``type`` (a name or a list of names), ``properties``,
    ``required``, ``additionalProperties`` (``false`` or a schema), ``items``,
    ``enum``, ``minimum``, ``maximum``. Anything else is ignored.
    """
    issues: list[str] = []
    _check(schema, value, "", issues)
    return issues


def _where(path: str) -> str:
    return path or "<root>"


def _check(schema: Any, value: Any, path: str, issues: list[str]) -> None:
    if not isinstance(schema, Mapping):
        return
    names = schema.get("type")
    names = [names] if isinstance(names, str) else [n for n in names or () if isinstance(n, str)]
    if names and not any(_TYPE_CHECKS.get(n, lambda _v: True)(value) for n in names):
        issues.append(f"Parameter `{_where(path)}` must be {' or '.join(names)}.")
        return
    if isinstance(value, Mapping):
        props = schema.get("properties")
        props = props if isinstance(props, Mapping) else {}
        required = [k for k in schema.get("required") or () if isinstance(k, str)]
        issues.extend(f"The required parameter `{_join(path, k)}` is missing." for k in required if k not in value)
        extra = schema.get("additionalProperties")
        if extra is False:
            issues.extend(f"Unexpected parameter `{_join(path, k)}`." for k in value if k not in props)
        for key, item in value.items():
            if key in props:
                _check(props[key], item, _join(path, key), issues)
            elif isinstance(extra, Mapping):
                _check(extra, item, _join(path, key), issues)
    if isinstance(value, list):
        for i, item in enumerate(value):
            _check(schema.get("items"), item, f"{path}[{i}]", issues)
    enum = schema.get("enum")
    if isinstance(enum, list | tuple) and value not in enum:
        allowed = ", ".join(repr(e) for e in enum)
        issues.append(f"Parameter `{_where(path)}` must be one of {allowed}.")
    if isinstance(value, int | float) and not isinstance(value, bool):
        lo, hi = schema.get("minimum"), schema.get("maximum")
        if isinstance(lo, int | float) and value < lo:
            issues.append(f"Parameter `{_where(path)}` must be >= {lo}.")
        if isinstance(hi, int | float) and value > hi:
            issues.append(f"Parameter `{_where(path)}` must be <= {hi}.")


def _join(path: str, key: str) -> str:
    return f"{path}.{key}" if path else key


# ---------------------------------------------------------------------------- coercion
_TRUE = frozenset({"true", "1", "yes", "y", "on"})
_FALSE = frozenset({"false", "0", "no", "n", "off", ""})


def bool_val(value: Any, default: bool = False) -> bool:
    """``bool`` from JSON-ish input; an unrecognised string gives ``default`` (``"false"`` is False)."""
    if isinstance(value, bool):
        return value
    if isinstance(value, int | float):
        return bool(value)
    if isinstance(value, str):
        word = value.strip().lower()
        if word in _TRUE:
            return True
        if word in _FALSE:
            return False
    return default


def _number(value: Any, cast: Callable[[Any], Any], default: Any) -> Any:
    if isinstance(value, bool):  # a JSON true where a number belongs is a shape error, not 1
        return default
    if isinstance(value, int | float):
        return cast(value)
    if isinstance(value, str):
        try:
            return cast(value.strip())
        except ValueError:
            return default
    return default


def float_val(value: Any, default: float = 0.0) -> float:
    """``float`` from a number or numeric string, else ``default`` (booleans are not numbers here)."""
    return _number(value, float, default)


def int_val(value: Any, default: int) -> int:
    """``int`` from a number (truncating) or an integer string, else ``default``."""
    return _number(value, int, default)


def str_val(value: Any, default: str = "") -> str:
    """A string as is; anything else (numbers included) is a shape mismatch and gives ``default``."""
    return value if isinstance(value, str) else default


def dict_val(value: Any, item: type = object) -> dict[str, Any]:
    """A mapping's entries whose values are ``item`` instances (all by default), keys as strings; else ``{}``."""
    if not isinstance(value, Mapping):
        return {}
    return {str(k): v for k, v in value.items() if isinstance(v, item)}


def list_val(value: Any, item: type = object) -> list[Any]:
    """A list's elements that are ``item`` instances (all by default); ``[]`` for anything but a list."""
    if not isinstance(value, list):
        return []
    return [v for v in value if isinstance(v, item)]


def dicts_val(value: Any) -> list[dict[str, Any]]:
    """The non-empty object elements of a list, each as a plain ``dict``."""
    return [d for v in list_val(value) if (d := dict_val(v))]


def datetime_val(value: Any, default: datetime | None = None) -> datetime | None:
    """A ``datetime`` parsed from an ISO 8601 string; ``default`` for anything else or a malformed string."""
    if not isinstance(value, str) or not value:
        return default
    try:
        return datetime.fromisoformat(value)
    except ValueError:
        return default


# ---------------------------------------------------------------------------- dataclass codec
class SchemaError(ValueError):
    """A JSON object does not fit the dataclass it is decoded into (a key names no field)."""


# special scalars: type -> (encode, decode) between the value and its JSON string/number
_SCALARS: dict[type, tuple[Callable[[Any], Any], Callable[[Any, Any], Any]]] = {
    bytes: (lambda v: base64.b64encode(v).decode("ascii"), lambda _t, raw: base64.b64decode(raw)),
    Path: (str, lambda _t, raw: Path(raw)),
    UUID: (str, lambda _t, raw: UUID(raw)),
    datetime: (lambda v: v.isoformat(), lambda _t, raw: datetime.fromisoformat(raw)),
    Enum: (lambda v: v.value, lambda t, raw: t(raw)),
}


def _scalar_kind(tp: Any) -> type | None:
    """The codec entry of a special scalar type (``Enum`` subclasses share one)."""
    if not isinstance(tp, type):
        return None
    for kind in _SCALARS:
        if issubclass(tp, kind):
            return kind
    return None


def _is_union(tp: Any) -> bool:
    return get_origin(tp) in (Union, types.UnionType)


def _resolve(tp: Any) -> Any:
    """Unwrap ``type X = ...`` aliases."""
    return getattr(tp, "__value__", tp) if type(tp).__name__ == "TypeAliasType" else tp


def _drop_none(tp: Any) -> Any:
    tp = _resolve(tp)
    if _is_union(tp):
        rest = [a for a in get_args(tp) if a is not type(None)]
        if len(rest) == 1:
            return rest[0]
    return tp


@cache
def _hints(cls: type) -> dict[str, Any]:
    return get_type_hints(cls)


@cache
def _init_fields(cls: type) -> frozenset[str]:
    return frozenset(f.name for f in fields(cls) if f.init)


def dataclass_to_json(obj: Any) -> dict[str, Any]:
    """Tagged JSON object of a dataclass instance (its ``init`` fields, recursively encoded)."""
    if not is_dataclass(obj) or isinstance(obj, type):
        raise TypeError(f"dataclass_to_json expects a dataclass instance, got {obj!r}")
    hints = _hints(type(obj))
    out: dict[str, Any] = {TYPE_TAG: type(obj).__name__}
    for f in fields(obj):
        if f.init:
            out[f.name] = _encode(getattr(obj, f.name), hints.get(f.name))
    return out


def _encode(value: Any, annotation: Any = None) -> Any:
    ann = _resolve(annotation)
    if is_dataclass(value) and not isinstance(value, type):
        return dataclass_to_json(value)
    kind = _scalar_kind(type(value))
    if kind is not None:
        encoded = _SCALARS[kind][0](value)
        if _is_union(ann) and sum(_scalar_kind(a) is not None for a in get_args(ann)) >= 2:
            return {SCALAR_TAG: type(value).__name__, VALUE_TAG: encoded}
        return encoded
    if value is None or isinstance(value, bool | int | float | str):
        return value
    if isinstance(value, Mapping):
        val_ann = _arg(ann, 1)
        return {str(k): _encode(v, val_ann) for k, v in value.items()}
    if isinstance(value, AbstractSet):
        elem = _arg(ann, 0)
        return sorted((_encode(v, elem) for v in value), key=repr)
    if isinstance(value, Sequence):
        anns = _elements(ann, len(value))
        return [_encode(v, a) for v, a in zip(value, anns, strict=True)]
    raise TypeError(f"cannot encode {type(value).__name__} to JSON")


def _arg(annotation: Any, i: int) -> Any:
    args = get_args(_drop_none(annotation))
    return args[i] if len(args) > i else None


def _elements(annotation: Any, n: int) -> list[Any]:
    ann = _drop_none(annotation)
    args = get_args(ann)
    if not args:
        return [None] * n
    if get_origin(ann) is tuple:
        if len(args) == 2 and args[1] is Ellipsis:
            return [args[0]] * n
        return list(args) if len(args) == n else [None] * n
    return [args[0]] * n


def dataclass_from_json(cls: type[T], data: Mapping[str, Any]) -> T:
    """Rebuild ``cls`` from a JSON object; its ``init`` parameters are the schema.

    Raises :class:`SchemaError` for keys that name no ``init`` field (a
    misspelt key must not silently fall back to the default). The ``__type__``
    tag is ignored: the caller chose ``cls``.
    """
    allowed = _init_fields(cls)
    unknown = sorted(k for k in data if k != TYPE_TAG and k not in allowed)
    if unknown:
        raise SchemaError(f"{cls.__name__}: unknown field(s) {unknown}; valid: {sorted(allowed)}")
    hints = _hints(cls)
    return cls(**{k: decode(hints.get(k), v) for k, v in data.items() if k != TYPE_TAG})


def decode(annotation: Any, raw: Any) -> Any:
    """A JSON value decoded against a type annotation (``None`` annotation: returned as is)."""
    ann = _resolve(annotation)
    if raw is None or ann is None or ann is Any:
        return raw
    if _is_union(ann):
        return _decode_union(ann, raw)
    if isinstance(ann, type) and is_dataclass(ann):
        if not isinstance(raw, Mapping):
            raise TypeError(f"expected an object for {ann.__name__}, got {raw!r}")
        return dataclass_from_json(ann, raw)
    origin = get_origin(ann)
    if origin in (list, tuple, set, frozenset, Sequence, AbstractSet) and isinstance(raw, list):
        items = [decode(a, v) for a, v in zip(_elements(ann, len(raw)), raw, strict=True)]
        if origin in (set, AbstractSet):
            return set(items)
        if origin is frozenset:
            return frozenset(items)
        return tuple(items) if origin in (tuple, Sequence) else items
    if origin in (dict, Mapping) and isinstance(raw, Mapping):
        val_ann = _arg(ann, 1)
        return {k: decode(val_ann, v) for k, v in raw.items()}
    kind = _scalar_kind(ann)
    if kind is not None:
        return _SCALARS[kind][1](ann, raw)
    if ann is bool:
        return bool_val(raw)
    if ann is int and not isinstance(raw, bool) and isinstance(raw, int | float | str):
        return int(float(raw)) if isinstance(raw, str) else int(raw)
    if ann is float and not isinstance(raw, bool) and isinstance(raw, int | float | str):
        return float(raw)
    if ann is str:
        if isinstance(raw, str):
            return raw
        if isinstance(raw, int | float) and not isinstance(raw, bool):
            return str(raw)
        raise TypeError(f"cannot read {raw!r} as a string")
    return raw


def _decode_union(ann: Any, raw: Any) -> Any:
    members = [a for a in get_args(ann) if a is not type(None)]
    if isinstance(raw, Mapping):
        tag = raw.get(TYPE_TAG)
        for m in members:
            if isinstance(m, type) and is_dataclass(m) and m.__name__ == tag:
                return dataclass_from_json(m, raw)
        name = raw.get(SCALAR_TAG)
        for m in members:
            if isinstance(name, str) and isinstance(m, type) and m.__name__ == name:
                return decode(m, raw.get(VALUE_TAG))
    if len(members) == 1:
        return decode(members[0], raw)
    for m in members:  # a JSON-native member that already fits the value
        if m in (bool, int, float, str) and isinstance(raw, m) and not (m is int and isinstance(raw, bool)):
            return raw
    for m in members:  # otherwise the first member that decodes it
        try:
            return decode(m, raw)
        except (TypeError, ValueError):
            continue
    return raw


class JsonCodec:
    """Mixin for dataclasses: ``to_json()`` and ``from_json(data)`` through the tagged codec."""

    def to_json(self) -> dict[str, Any]:
        return dataclass_to_json(self)

    @classmethod
    def from_json(cls: type[T], data: Mapping[str, Any]) -> T:
        return dataclass_from_json(cls, data)
