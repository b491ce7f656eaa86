"""Bit-for-bit golden tests (``priml/testing/bfb.py:384-990``).

Pattern: build a module at minimal width, randomize every parameter (so
structurally-zero inits cannot hide a regression), run it on a fixed input and
store ``(state before, input, output, state after)`` under ``golden_dir``;
later runs must reproduce the output and the post-run state with
``torch.equal``. ``BFB_REGENERATE=1`` rewrites the goldens after an
intentional numeric change.

Portability across hosts comes from :func:`host_agnostic_numerics`, a dispatch
mode that runs every float32 arithmetic op in float64 and rounds the result to
float32 once: a float64 accumulation rounded to float32 no longer depends on the
host's vector width or thread count. View / metadata ops pass through
untouched; in-place and ``out=`` ops are computed in float64 and written back.
Goldens are CPU-only: GPU kernel selection and reduction order differ across
GPU models.
"""

from __future__ import annotations

import os
from collections.abc import Callable, Iterator
from contextlib import contextmanager
from pathlib import Path
from typing import Any

import torch
from torch import Tensor, nn
from torch.utils._python_dispatch import TorchDispatchMode
from torch.utils._pytree import tree_map

__all__ = [
    "assert_bfb_against_golden",
    "bfb_devices",
    "host_agnostic_numerics",
    "move_to_device",
    "randomize_parameters",
    "regenerate_golden",
]

_aten = torch.ops.aten
# Ops whose float32 result is already exact / host independent: data movement and creation.
_PASS_THROUGH = {
    _aten.clone.default, _aten.copy_.default, _aten.detach.default, _aten._to_copy.default, _aten.cat.default,
    _aten.stack.default, _aten.index.Tensor, _aten.index_select.default, _aten.gather.default,
    _aten.embedding.default, _aten.fill_.Scalar, _aten.zero_.default, _aten.empty_like.default,
    _aten.zeros_like.default, _aten.ones_like.default, _aten.full_like.default, _aten.where.self,
    _aten.masked_fill.Scalar, _aten.masked_fill_.Scalar, _aten.lift_fresh.default, _aten.constant_pad_nd.default,
    _aten.flip.default, _aten.roll.default, _aten.repeat.default, _aten.split_with_sizes.default,
    _aten.unbind.int, _aten.split.Tensor, _aten.chunk.default, _aten.neg.default, _aten.abs.default,
    _aten.relu.default, _aten.max.dim, _aten.amax.default, _aten.argmax.default, _aten.sort.default,
}  # fmt: skip


def _is_f32(x: Any) -> bool:
    return isinstance(x, Tensor) and x.dtype == torch.float32


class _Float64Mode(TorchDispatchMode):
    def __torch_dispatch__(self, func, types, args=(), kwargs=None):  # noqa: ANN001, ANN204
        kwargs = kwargs or {}
        flat = [*args, *kwargs.values()]
        if func in _PASS_THROUGH or getattr(func, "is_view", False) or not any(
            _is_f32(a) or (isinstance(a, (list, tuple)) and any(_is_f32(t) for t in a)) for a in flat
        ):
            return func(*args, **kwargs)
        up = tree_map(lambda a: a.to(torch.float64) if _is_f32(a) else a, (args, kwargs))
        out = func(*up[0], **up[1])
        schema = func._schema  # noqa: SLF001
        mutated = [i for i, arg in enumerate(schema.arguments) if arg.alias_info is not None and arg.alias_info.is_write]
        if mutated:
            # write float64 results back into the original float32 storage
            names = [schema.arguments[i].name for i in mutated]
            for i, name in zip(mutated, names, strict=True):
                orig = args[i] if i < len(args) else kwargs.get(name)
                new = up[0][i] if i < len(up[0]) else up[1].get(name)
                if _is_f32(orig):
                    orig.copy_(new.to(torch.float32))
            result_list = out if isinstance(out, (tuple, list)) else (out,)
            fixed = []
            for r in result_list:
                src = None
                for i, name in zip(mutated, names, strict=True):
                    new = up[0][i] if i < len(up[0]) else up[1].get(name)
                    if r is new:
                        src = args[i] if i < len(args) else kwargs.get(name)
                fixed.append(src if src is not None else (r.to(torch.float32) if isinstance(r, Tensor) and r.dtype == torch.float64 else r))
            return type(out)(fixed) if isinstance(out, (tuple, list)) else fixed[0]
        return tree_map(lambda r: r.to(torch.float32) if isinstance(r, Tensor) and r.dtype == torch.float64 else r, out)


@contextmanager
def host_agnostic_numerics() -> Iterator[None]:
    """Run the wrapped float32 computation in float64, rounding each op's result to float32."""
    with _Float64Mode():
        yield


def bfb_devices() -> list[str]:
    return ["cpu"]


def move_to_device(value: Any, device: str | torch.device) -> Any:
    if isinstance(value, Tensor):
        return value.to(device)
    if isinstance(value, dict):
        return {k: move_to_device(v, device) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return type(value)(move_to_device(v, device) for v in value)
    return value


def randomize_parameters(module: nn.Module, *, seed: int, std: float = 1.0) -> None:
    """Overwrite every parameter with ``N(0, std^2)`` from a private generator (buffers untouched)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for p in module.parameters():
            p.copy_((torch.randn(p.shape, generator=g, dtype=torch.float64) * std).to(p.dtype))


def _default_run(module: nn.Module, inputs: Any) -> Any:
    if isinstance(inputs, dict):
        return module(**inputs)
    if isinstance(inputs, (tuple, list)):
        return module(*inputs)
    return module(inputs)


def _execute(module: nn.Module, inputs: Any, run: Callable[[nn.Module, Any], Any] | None) -> Any:
    with host_agnostic_numerics():
        out = (run or _default_run)(module, inputs)
    return tree_map(lambda t: t.detach().clone() if isinstance(t, Tensor) else t, out)


def _state(module: nn.Module) -> dict[str, Tensor]:
    return {k: v.detach().clone() for k, v in module.state_dict().items()}


def _equal(a: Any, b: Any) -> bool:
    if isinstance(a, Tensor) and isinstance(b, Tensor):
        return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)
    if isinstance(a, dict) and isinstance(b, dict):
        return a.keys() == b.keys() and all(_equal(a[k], b[k]) for k in a)
    if isinstance(a, (list, tuple)) and isinstance(b, (list, tuple)):
        return len(a) == len(b) and all(_equal(x, y) for x, y in zip(a, b, strict=True))
    return a == b


def regenerate_golden(*, golden_dir: Path | str, golden_name: str, build_module: Callable[[], nn.Module],
                      build_input: Callable[[], Any], seed: int = 0,
                      run: Callable[[nn.Module, Any], Any] | None = None) -> Path:  # fmt: skip
    path = Path(golden_dir) / f"{golden_name}.pt"
    path.parent.mkdir(parents=True, exist_ok=True)
    module = build_module()
    inputs = build_input()
    randomize_parameters(module, seed=seed)
    before = _state(module)
    output = _execute(module, inputs, run)
    torch.save({"state": before, "input": inputs, "output": output, "post_state": _state(module)}, path)
    _replay(path, build_module, run)
    return path


def _replay(path: Path, build_module: Callable[[], nn.Module], run: Callable[[nn.Module, Any], Any] | None) -> None:
    golden = torch.load(path, map_location="cpu", weights_only=False)
    module = build_module()
    module.load_state_dict(golden["state"])
    output = _execute(module, golden["input"], run)
    if not _equal(output, golden["output"]):
        raise AssertionError(f"output differs from golden {path}")
    if not _equal(_state(module), golden["post_state"]):
        raise AssertionError(f"post-run state differs from golden {path}")


def assert_bfb_against_golden(*, golden_dir: Path | str, golden_name: str, build_module: Callable[[], nn.Module],
                              build_input: Callable[[], Any], seed: int = 0,
                              run: Callable[[nn.Module, Any], Any] | None = None) -> None:  # fmt: skip
    """Replay the golden (writing it first when missing or when ``BFB_REGENERATE=1``)."""
    path = Path(golden_dir) / f"{golden_name}.pt"
    if os.environ.get("BFB_REGENERATE") == "1" or not path.exists():
        regenerate_golden(golden_dir=golden_dir, golden_name=golden_name, build_module=build_module,
                          build_input=build_input, seed=seed, run=run)  # fmt: skip
        return
    _replay(path, build_module, run)
