"""Config trees: typed, nestable, finalizable configs that build objects.

The reference builds every object from a tree of ``Fig`` configs
(``from configgle import Fig, Makeable, Makes, PartialConfig, ...``; e.g.
``priml/model/causal_lm.py:49``, ``priml/launch.py:102-125``). That library is
not installable offline, so this package provides the same public surface:

* ``Fig["Target"]`` -- base of a nested ``Config`` dataclass whose ``make()``
  builds ``Target(finalized_config)``. ``kw_only`` is a class keyword.
* ``Makes["Other"]`` -- mixin that re-targets an inherited ``Config``.
* ``PartialConfig(fn, *a, **kw)`` -- ``make()`` returns ``functools.partial``.
* ``InlineConfig(fn, *a, **kw)`` -- ``make()`` calls ``fn(*a, **kw)``.
* ``Makeable[T]`` / ``Maker`` -- the "has ``make()``" protocol.
* ``MutableNamespace`` -- attribute bag that participates in copy/pformat.
* ``finalize`` / ``copy_tree`` / ``pformat`` / ``pprint`` on every config, and
  the free functions ``copy_tree``, ``apply_overrides``, ``resolve_config``.

Semantics chosen here (documented because the original is closed to us):

* ``finalize()`` is the place where parents push shared values into children
  (``propagate_attr``); the base implementation finalizes every child config
  and then freezes the node. Mutating a frozen node raises
  ``dataclasses.FrozenInstanceError``; ``object.__setattr__`` bypasses it.
* ``make()`` always works on a fresh, unfrozen ``copy_tree()`` of the receiver
  and finalizes that copy, so the same template can be made many times (with
  e.g. a different ``depth`` written into it) and propagation re-runs.
"""

from __future__ import annotations

import copy
import dataclasses
import functools
import importlib
import json
import sys
import types
import typing
from collections.abc import Callable, Iterable
from typing import Any, Generic, Protocol, TypeVar, runtime_checkable

__all__ = [
    "Fig",
    "InlineConfig",
    "Makeable",
    "Maker",
    "Makes",
    "MutableNamespace",
    "PartialConfig",
    "apply_overrides",
    "copy_tree",
    "finalize",
    "pformat",
    "pprint",
    "resolve_config",
]

T = TypeVar("T", covariant=True)


@runtime_checkable
class Maker(Protocol):
    """Anything with a ``make()`` method."""

    def make(self) -> Any: ...


class _MakeableAlias:
    """``Makeable[T]`` is a typing-only alias of :class:`Maker`."""

    def __getitem__(self, item: Any) -> Any:
        return Maker

    def __instancecheck__(self, obj: Any) -> bool:
        return isinstance(obj, Maker)


Makeable: Any = _MakeableAlias()


def _is_config(obj: Any) -> bool:
    return isinstance(obj, (_FigBase, PartialConfig, InlineConfig, MutableNamespace))


# --------------------------------------------------------------------------------------
# Fig
# --------------------------------------------------------------------------------------


class _FigBase:
    """Behaviour shared by every ``Fig`` config dataclass."""

    _fig_target_name: typing.ClassVar[str | None] = None
    _fig_target_cache: typing.ClassVar[Any] = None

    def __init_subclass__(cls, kw_only: bool = True, **kwargs: Any) -> None:
        super().__init_subclass__(**kwargs)
        # Skip the anonymous Fig["X"] / Makes["X"] carrier classes.
        if cls.__dict__.get("_fig_carrier", False):
            return
        cls._fig_target_cache = None
        dataclasses.dataclass(kw_only=kw_only, eq=True, repr=False)(cls)

    # ---- freezing -------------------------------------------------------------------
    def __setattr__(self, name: str, value: Any) -> None:
        if self.__dict__.get("_fig_frozen", False) and not name.startswith("_fig"):
            raise dataclasses.FrozenInstanceError(
                f"cannot assign to field {name!r} of finalized {type(self).__qualname__}"
            )
        object.__setattr__(self, name, value)

    @property
    def is_finalized(self) -> bool:
        return bool(self.__dict__.get("_fig_frozen", False))

    # ---- tree ops -------------------------------------------------------------------
    def finalize(self):  # noqa: ANN201 - returns Self
        """Finalize children, then freeze this node. Subclasses push values down
        into children *before* calling ``super().finalize()``."""
        if self.is_finalized:
            return self
        for f in dataclasses.fields(self):  # type: ignore[arg-type]
            value = getattr(self, f.name)
            object.__setattr__(self, f.name, _finalize_value(value))
        object.__setattr__(self, "_fig_frozen", True)
        return self

    def copy_tree(self):  # noqa: ANN201 - returns Self
        """Deep copy of this config tree, with every node unfrozen."""
        return copy_tree(self)

    def make(self) -> Any:
        """Build the target object from a finalized copy of this config."""
        cfg = self.copy_tree().finalize()
        target = type(self)._resolve_target()
        return target(cfg)

    @classmethod
    def _resolve_target(cls) -> Any:
        if cls._fig_target_cache is not None:
            return cls._fig_target_cache
        name = None
        for klass in cls.__mro__:
            name = klass.__dict__.get("_fig_target_name")
            if name:
                break
        if not name:
            raise TypeError(f"{cls.__qualname__} has no Fig target")
        target = _lookup_target(cls, name)
        cls._fig_target_cache = target
        return target

    # ---- printing -------------------------------------------------------------------
    def pformat(self, *, finalize: bool = False, hide_default_values: bool = True) -> str:
        node = self.copy_tree().finalize() if finalize else self
        return _pformat(node, 0, hide_default_values)

    def pprint(self, *, finalize: bool = False, hide_default_values: bool = True) -> None:
        print(self.pformat(finalize=finalize, hide_default_values=hide_default_values))

    def __repr__(self) -> str:
        return self.pformat(hide_default_values=True)

    def __deepcopy__(self, memo: dict[int, Any]) -> Any:
        new = object.__new__(type(self))
        memo[id(self)] = new
        for k, v in self.__dict__.items():
            if k == "_fig_frozen":
                continue
            object.__setattr__(new, k, copy.deepcopy(v, memo) if _copyable(v) else v)
        return new


def _copyable(v: Any) -> bool:
    # Functions, classes, modules, dtypes and devices are shared, not copied.
    return not isinstance(
        v,
        (types.FunctionType, types.BuiltinFunctionType, type, types.ModuleType, functools.partial),
    ) and not _is_torch_atom(v)


def _is_torch_atom(v: Any) -> bool:
    mod = type(v).__module__
    return mod == "torch" and type(v).__name__ in ("dtype", "device", "memory_format", "layout")


def _lookup_target(cls: type, name: str) -> Any:
    module = sys.modules.get(cls.__module__)
    # Enclosing class first: "Outer.Config" targets "Outer".
    qual = cls.__qualname__.split(".")
    if len(qual) >= 2 and module is not None:
        obj: Any = module
        ok = True
        for part in qual[:-1]:
            if part == "<locals>":
                ok = False
                break
            obj = getattr(obj, part, None)
            if obj is None:
                ok = False
                break
        if ok and getattr(obj, "__name__", None) == name.split(".")[-1]:
            return obj
    if module is not None:
        obj = module
        for part in name.split("."):
            obj = getattr(obj, part, None)
            if obj is None:
                break
        if obj is not None:
            return obj
    # Fully qualified "pkg.mod.Name".
    if "." in name:
        mod_name, attr = name.rsplit(".", 1)
        return getattr(importlib.import_module(mod_name), attr)
    raise LookupError(f"cannot resolve Fig target {name!r} for {cls.__qualname__}")


class _FigMeta(type):
    def __getitem__(cls, name: str) -> type:
        carrier = type(
            f"{cls.__name__}[{name}]",
            (_FigBase,),
            {"_fig_carrier": True, "_fig_target_name": name, "__module__": __name__},
        )
        return carrier


class Fig(metaclass=_FigMeta):
    """``class Config(Fig["Target"], kw_only=False): ...`` -- see module doc."""


class Makes(metaclass=_FigMeta):
    """``class Config(Makes["Other"], Base.Config): ...`` re-targets ``make()``."""


# --------------------------------------------------------------------------------------
# Partial / Inline configs
# --------------------------------------------------------------------------------------


class _CallConfig:
    """Shared body of PartialConfig and InlineConfig: a callable plus arguments,
    with keyword arguments readable/writable as attributes."""

    def __init__(self, fn: Callable[..., Any], /, *args: Any, **kwargs: Any) -> None:
        object.__setattr__(self, "_fn", fn)
        object.__setattr__(self, "_args", list(args))
        object.__setattr__(self, "_kwargs", dict(kwargs))
        object.__setattr__(self, "_fig_frozen", False)

    @property
    def fn(self) -> Callable[..., Any]:
        return self._fn

    @property
    def args(self) -> tuple[Any, ...]:
        return tuple(self._args)

    @property
    def kwargs(self) -> dict[str, Any]:
        return dict(self._kwargs)

    def __getattr__(self, name: str) -> Any:
        kwargs = self.__dict__.get("_kwargs", {})
        if name in kwargs:
            return kwargs[name]
        raise AttributeError(name)

    def __setattr__(self, name: str, value: Any) -> None:
        if name.startswith("_"):
            object.__setattr__(self, name, value)
            return
        if self.__dict__.get("_fig_frozen", False):
            raise dataclasses.FrozenInstanceError(f"cannot assign {name!r} on finalized config")
        self._kwargs[name] = value

    def __hasattr_kw__(self, name: str) -> bool:
        return name in self._kwargs

    @property
    def is_finalized(self) -> bool:
        return bool(self.__dict__.get("_fig_frozen", False))

    def finalize(self):  # noqa: ANN201
        if self.is_finalized:
            return self
        object.__setattr__(self, "_args", [_finalize_value(a) for a in self._args])
        object.__setattr__(self, "_kwargs", {k: _finalize_value(v) for k, v in self._kwargs.items()})
        object.__setattr__(self, "_fig_frozen", True)
        return self

    def copy_tree(self):  # noqa: ANN201
        return copy_tree(self)

    def _made_args(self) -> tuple[list[Any], dict[str, Any]]:
        args = [_make_value(a) for a in self._args]
        kwargs = {k: _make_value(v) for k, v in self._kwargs.items()}
        return args, kwargs

    def __deepcopy__(self, memo: dict[int, Any]) -> Any:
        new = object.__new__(type(self))
        memo[id(self)] = new
        object.__setattr__(new, "_fn", self._fn)
        object.__setattr__(new, "_args", [copy.deepcopy(a, memo) if _copyable(a) else a for a in self._args])
        object.__setattr__(
            new, "_kwargs", {k: (copy.deepcopy(v, memo) if _copyable(v) else v) for k, v in self._kwargs.items()}
        )
        object.__setattr__(new, "_fig_frozen", False)
        return new

    def __eq__(self, other: object) -> bool:
        return (
            type(other) is type(self)
            and self._fn is other._fn  # type: ignore[attr-defined]
            and self._args == other._args  # type: ignore[attr-defined]
            and self._kwargs == other._kwargs  # type: ignore[attr-defined]
        )

    __hash__ = None  # type: ignore[assignment]

    def pformat(self, *, finalize: bool = False, hide_default_values: bool = True) -> str:
        return _pformat(self, 0, hide_default_values)

    def __repr__(self) -> str:
        return self.pformat()


class PartialConfig(_CallConfig):
    """``make()`` returns ``functools.partial(fn, *args, **kwargs)`` (nested
    configs among the arguments are made first)."""

    def make(self) -> Any:
        cfg = self.copy_tree().finalize()
        args, kwargs = cfg._made_args()
        return functools.partial(cfg._fn, *args, **kwargs)


class InlineConfig(_CallConfig):
    """``make()`` returns ``fn(*args, **kwargs)``."""

    def make(self) -> Any:
        cfg = self.copy_tree().finalize()
        args, kwargs = cfg._made_args()
        return cfg._fn(*args, **kwargs)


class MutableNamespace(types.SimpleNamespace):
    """Attribute bag that copies, finalizes and prints like a config node."""

    def finalize(self):  # noqa: ANN201
        for k, v in list(vars(self).items()):
            setattr(self, k, _finalize_value(v))
        return self

    def copy_tree(self):  # noqa: ANN201
        return copy_tree(self)

    def make(self) -> Any:
        return self


# --------------------------------------------------------------------------------------
# tree helpers
# --------------------------------------------------------------------------------------


def _finalize_value(value: Any) -> Any:
    if isinstance(value, (_FigBase, _CallConfig, MutableNamespace)):
        return value.finalize()
    if isinstance(value, list):
        return [_finalize_value(v) for v in value]
    if isinstance(value, tuple) and not hasattr(value, "_fields"):
        return tuple(_finalize_value(v) for v in value)
    if isinstance(value, dict):
        return {k: _finalize_value(v) for k, v in value.items()}
    return value


def _make_value(value: Any) -> Any:
    if isinstance(value, (_FigBase, _CallConfig)):
        return value.make()
    return value


def finalize(config: Any) -> Any:
    """Finalize ``config`` (free-function form)."""
    return config.finalize()


def copy_tree(config: Any) -> Any:
    """Deep copy a config tree; every copied node is unfrozen."""
    return copy.deepcopy(config)


def _field_default(f: dataclasses.Field[Any]) -> Any:
    if f.default is not dataclasses.MISSING:
        return f.default
    if f.default_factory is not dataclasses.MISSING:  # type: ignore[misc]
        try:
            return f.default_factory()  # type: ignore[misc]
        except Exception:  # noqa: BLE001
            return dataclasses.MISSING
    return dataclasses.MISSING


def _fmt_atom(v: Any) -> str:
    if isinstance(v, (types.FunctionType, types.BuiltinFunctionType)):
        return f"{getattr(v, '__module__', '?')}.{getattr(v, '__qualname__', repr(v))}"
    if isinstance(v, type):
        return f"{v.__module__}.{v.__qualname__}"
    if isinstance(v, functools.partial):
        return f"partial({_fmt_atom(v.func)}, ...)"
    return repr(v)


def _pformat(node: Any, indent: int, hide_defaults: bool) -> str:
    pad = "  " * (indent + 1)
    if isinstance(node, _FigBase):
        lines = [f"{type(node).__qualname__}("]
        for f in dataclasses.fields(node):  # type: ignore[arg-type]
            if f.name == "_":
                continue
            v = getattr(node, f.name)
            if hide_defaults:
                d = _field_default(f)
                try:
                    same = d is not dataclasses.MISSING and bool(d == v)
                except Exception:  # noqa: BLE001
                    same = False
                if same:
                    continue
            lines.append(f"{pad}{f.name}={_pformat(v, indent + 1, hide_defaults)},")
        lines.append("  " * indent + ")")
        return "\n".join(lines) if len(lines) > 2 else f"{type(node).__qualname__}()"
    if isinstance(node, _CallConfig):
        parts = [_fmt_atom(node._fn)]
        parts += [_pformat(a, indent + 1, hide_defaults) for a in node._args]
        parts += [f"{k}={_pformat(v, indent + 1, hide_defaults)}" for k, v in node._kwargs.items()]
        return f"{type(node).__name__}({', '.join(parts)})"
    if isinstance(node, list):
        if not node:
            return "[]"
        inner = [f"{pad}{_pformat(v, indent + 1, hide_defaults)}," for v in node]
        return "[\n" + "\n".join(inner) + "\n" + "  " * indent + "]"
    return _fmt_atom(node)


def pformat(config: Any, *, finalize: bool = False, hide_default_values: bool = True) -> str:
    return config.pformat(finalize=finalize, hide_default_values=hide_default_values)


def pprint(config: Any, *, finalize: bool = False, hide_default_values: bool = True) -> None:
    print(pformat(config, finalize=finalize, hide_default_values=hide_default_values))


# --------------------------------------------------------------------------------------
# overrides / launch
# --------------------------------------------------------------------------------------


def _parse_value(text: str) -> Any:
    try:
        return json.loads(text)
    except (json.JSONDecodeError, ValueError):
        low = text.lower()
        if low in ("true", "false"):
            return low == "true"
        if low in ("none", "null"):
            return None
        if low in ("inf", "+inf"):
            return float("inf")
        return text


def _cast_to(annotation: Any, value: Any, current: Any) -> Any:
    if value is None:
        return None
    if isinstance(current, bool) or annotation is bool:
        return bool(value)
    if isinstance(current, int) and not isinstance(current, bool) and isinstance(value, (int, float)):
        return int(value) if float(value).is_integer() else value
    if isinstance(current, float) and isinstance(value, (int, float)):
        return float(value)
    if isinstance(current, tuple) and isinstance(value, list):
        return tuple(value)
    if _is_torch_atom(current) and isinstance(value, str):
        import torch

        return getattr(torch, value.removeprefix("torch.")) if "dtype" in type(current).__name__ else torch.device(value)
    return value


def _set_path(config: Any, path: str, raw: Any) -> None:
    parts = path.split(".")
    node = config
    for part in parts[:-1]:
        if isinstance(node, list):
            node = node[int(part)]
        elif isinstance(node, dict):
            node = node[part]
        else:
            node = getattr(node, part)
    last = parts[-1]
    if isinstance(node, list):
        idx = int(last)
        node[idx] = _cast_to(None, raw, node[idx])
        return
    if isinstance(node, dict):
        node[last] = _cast_to(None, raw, node.get(last))
        return
    current = getattr(node, last, None)
    annotation = None
    if isinstance(node, _FigBase):
        names = {f.name: f for f in dataclasses.fields(node)}  # type: ignore[arg-type]
        if last not in names:
            raise AttributeError(f"{type(node).__qualname__} has no field {last!r}")
        annotation = names[last].type
    setattr(node, last, _cast_to(annotation, raw, current))


def apply_overrides(config: Any, overrides: Iterable[str]) -> Any:
    """Apply ``PATH=VALUE`` overrides in place. VALUE is JSON-parsed when it
    parses, else taken as a string; it is cast to the current field's type."""
    for item in overrides:
        if "=" not in item:
            raise ValueError(f"override {item!r} is not PATH=VALUE")
        path, text = item.split("=", 1)
        _set_path(config, path.strip(), _parse_value(text.strip()))
    return config


def resolve_config(spec: str) -> Any:
    """``"pkg.module.fn"`` -> ``fn()`` (or the attribute itself when it is a config)."""
    module_name, attr = spec.rsplit(".", 1)
    obj = getattr(importlib.import_module(module_name), attr)
    if callable(obj) and not _is_config(obj) and not isinstance(obj, type):
        return obj()
    if isinstance(obj, type) and issubclass(obj, _FigBase):
        return obj()
    return obj


# Generic re-export so ``Makeable[nn.Module]`` style annotations evaluate.
_ = Generic
