"""Route named parameters to member optimizers (``priml/optimizers/composite.py:39-468``).

Selectors are comparable objects (``everything``, ``matching``, ``excluding``,
``complement``) so configs holding them compare equal. A parameter may belong
to one member only; ``require_total`` rejects unclaimed parameters. State dict
is ``{"optimizers": [member_state, ...]}``.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator, MutableMapping, Sequence
from dataclasses import field
from functools import partial
from typing import Any, Protocol

from torch import nn
from torch.nn import Parameter
from torch.optim import Optimizer

from priml_b200.config import Fig

__all__ = ["CompositeOptimizer", "complement", "everything", "excluding", "matching"]


def everything(name: str, parameter: Parameter) -> bool:
    del name, parameter
    return True


def _name(sel: Any) -> str:
    q = getattr(sel, "__qualname__", None)
    return q if isinstance(q, str) else repr(sel)



class Selector(Protocol):
    """Whether one named parameter belongs to a member optimizer of a composite."""

    def __call__(self, name: str, parameter: Any) -> bool: ...

class excluding:  # noqa: N801
    __slots__ = ("fragments", "select")

    def __init__(self, select: Callable[[str, Parameter], bool], *fragments: str) -> None:
        self.select = select
        self.fragments = fragments

    def __call__(self, name: str, parameter: Parameter) -> bool:
        return self.select(name, parameter) and not any(f in name for f in self.fragments)

    def __eq__(self, other: object) -> bool:
        return isinstance(other, excluding) and self.select == other.select and self.fragments == other.fragments

    def __hash__(self) -> int:
        return hash((excluding, self.select, self.fragments))

    def __repr__(self) -> str:
        return f"excluding({_name(self.select)}, {', '.join(map(repr, self.fragments))})"


class matching:  # noqa: N801
    __slots__ = ("fragments",)

    def __init__(self, *fragments: str) -> None:
        self.fragments = fragments

    def __call__(self, name: str, parameter: Parameter) -> bool:
        del parameter
        return any(f in name for f in self.fragments)

    def __eq__(self, other: object) -> bool:
        return isinstance(other, matching) and self.fragments == other.fragments

    def __hash__(self) -> int:
        return hash((matching, self.fragments))

    def __repr__(self) -> str:
        return f"matching({', '.join(map(repr, self.fragments))})"


class complement:  # noqa: N801
    __slots__ = ("select",)

    def __init__(self, select: Callable[[str, Parameter], bool]) -> None:
        self.select = select

    def __call__(self, name: str, parameter: Parameter) -> bool:
        return not self.select(name, parameter)

    def __eq__(self, other: object) -> bool:
        return isinstance(other, complement) and self.select == other.select

    def __hash__(self) -> int:
        return hash((complement, self.select))

    def __repr__(self) -> str:
        return f"complement({_name(self.select)})"


class _ChainedState(MutableMapping):
    def __init__(self, optimizers: Sequence[Optimizer]) -> None:
        self._opts = optimizers

    def _owner(self, key: Any) -> dict:
        for o in self._opts:
            if key in o.state:
                return o.state
        return self._opts[0].state

    def __getitem__(self, key: Any) -> Any:
        for o in self._opts:
            if key in o.state:
                return o.state[key]
        raise KeyError(key)

    def __setitem__(self, key: Any, value: Any) -> None:
        self._owner(key)[key] = value

    def __delitem__(self, key: Any) -> None:
        del self._owner(key)[key]

    def __iter__(self) -> Iterator[Any]:
        for o in self._opts:
            yield from o.state

    def __len__(self) -> int:
        return sum(len(o.state) for o in self._opts)


def _reject_shared(optimizers: Sequence[Optimizer]) -> None:
    seen: dict[int, int] = {}
    for i, o in enumerate(optimizers):
        for g in o.param_groups:
            for p in g["params"]:
                if id(p) in seen and seen[id(p)] != i:
                    raise ValueError("A parameter appears in more than one member optimizer.")
                seen[id(p)] = i


def _route(
    model: nn.Module,
    members: Sequence[Callable[..., Optimizer]],
    selectors: Sequence[Callable[[str, Parameter], bool]],
    *,
    require_total: bool,
    drop_empty: bool = False,
) -> list[Optimizer]:
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    claimed: dict[int, str] = {}
    out: list[Optimizer] = []
    for member, select in zip(members, selectors, strict=True):
        group = []
        for name, p in named:
            if not select(name, p):
                continue
            if id(p) in claimed:
                raise ValueError(f"Parameter {name!r} is claimed by {claimed[id(p)]} and {_name(select)}.")
            claimed[id(p)] = _name(select)
            group.append(p)
        if not group:
            if drop_empty:
                continue
            raise ValueError(f"Selector {_name(select)} claims no parameter.")
        out.append(member(group))
    if require_total:
        missing = [n for n, p in named if id(p) not in claimed]
        if missing:
            raise ValueError(f"Parameters claimed by no member: {missing[:8]}")
    return out


class CompositeOptimizer(Optimizer):
    class Config(Fig["Callable[..., CompositeOptimizer]"]):
        optimizers: list[Any] = field(default_factory=list)
        select: list[Any] = field(default_factory=list)
        require_total: bool = True
        drop_empty: bool = False

        def make(self) -> Callable[..., CompositeOptimizer]:
            f = self.copy_tree().finalize()
            if not f.optimizers:
                raise ValueError("CompositeOptimizer.Config needs a member.")
            if f.select and len(f.select) != len(f.optimizers):
                raise ValueError(f"select names {len(f.select)} selectors for {len(f.optimizers)} optimizers.")
            members = [m.make() for m in f.optimizers]
            selectors = f.select or [everything] * len(members)
            req, drop = f.require_total, f.drop_empty

            def compose(model: nn.Module) -> CompositeOptimizer:
                return CompositeOptimizer(_route(model, members, selectors, require_total=req, drop_empty=drop))

            return partial(compose)

    def __init__(self, optimizers: Sequence[Optimizer]) -> None:  # noqa: D107 -- no super().__init__: groups are the members'
        if not optimizers:
            raise ValueError("CompositeOptimizer requires at least one optimizer.")
        _reject_shared(optimizers)
        self.optimizers = list(optimizers)
        self.defaults: dict[str, Any] = {}
        self.param_groups = [g for o in self.optimizers for g in o.param_groups]
        self.state = _ChainedState(self.optimizers)  # type: ignore[assignment]
        self._optimizer_step_pre_hooks: dict = {}
        self._optimizer_step_post_hooks: dict = {}

    def step(self, closure: Callable[[], Any] | None = None) -> Any:  # type: ignore[override]
        loss = closure() if closure is not None else None
        for o in self.optimizers:
            if closure is not None and getattr(o, "requires_closure", False):
                o.step(closure)
            else:
                o.step()
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        for o in self.optimizers:
            o.zero_grad(set_to_none=set_to_none)

    def state_dict(self) -> dict[str, Any]:
        return {"optimizers": [o.state_dict() for o in self.optimizers]}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        saved = state_dict["optimizers"]
        if len(saved) != len(self.optimizers):
            raise ValueError(f"Checkpoint holds {len(saved)} optimizers, composite has {len(self.optimizers)}.")
        for o, s in zip(self.optimizers, saved, strict=True):
            o.load_state_dict(s)
        self.param_groups = [g for o in self.optimizers for g in o.param_groups]

    def add_param_group(self, param_group: dict[str, Any]) -> None:
        del param_group
        raise NotImplementedError("Add the group to a member optimizer instead.")

    def __repr__(self) -> str:
        return f"CompositeOptimizer({', '.join(type(o).__name__ for o in self.optimizers)})"
