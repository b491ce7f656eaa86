"""DTensor tensor parallelism driven by shard styles declared on configs
(``priml/train/tensor_parallel.py:101-224``, ``priml/model/linear.py:154-199``,
``priml/model/swiglu.py:255-278``, ``priml/model/mla.py:590-622``).

Every building block declares ``shard in {colwise, rowwise, vocab}`` or supplies
its own ``tensor_parallel_style()``; :func:`apply_tensor_parallel` turns those
into one ``parallelize_module`` plan over the ``tp`` mesh axis. A ``tp`` size
of 1 is a structural no-op. This path runs the decomposed (DTensor) ops and is
the CPU/gloo-testable baseline; the fused AG-GEMM / GEMM-RS kernels of
:mod:`priml_b200.parallel.tp_fused` run the same sharding on local shards.
"""

from __future__ import annotations

import logging
from functools import partial
from typing import Any

import torch
from torch import nn
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.tensor import DTensor, Replicate, Shard, distribute_tensor
from torch.distributed.tensor.parallel import ColwiseParallel, ParallelStyle, RowwiseParallel, parallelize_module

from priml_b200.config import Fig
from priml_b200.parallel.runtime import global_device_mesh
from priml_b200.parallel.strategies import place

__all__ = ["EnsembleParallel", "MLAParallel", "SwiGLUParallel", "TensorParallel", "apply_tensor_parallel"]

log = logging.getLogger(__name__)


def _replicate_input(mesh: DeviceMesh, module: nn.Module, inputs: tuple[Any, ...]) -> tuple[Any, ...]:
    del module
    x = inputs[0]
    if isinstance(x, DTensor):
        x = x.redistribute(mesh, [Replicate()])
    else:
        x = DTensor.from_local(x, mesh, [Replicate()], run_check=False)
    return (x, *inputs[1:])


class EnsembleParallel(ParallelStyle):
    """Shard an ``[E, out, in]`` ensemble weight on E; replicate the input; the
    output stays a DTensor sharded on the ensemble dim."""

    def _apply(self, module: nn.Module, device_mesh: DeviceMesh) -> nn.Module:
        for name, p in list(module.named_parameters(recurse=False)):
            module.register_parameter(name, nn.Parameter(distribute_tensor(p, device_mesh, [Shard(0)])))
        module.register_forward_pre_hook(partial(_replicate_input, device_mesh))
        return module


class SwiGLUParallel(ParallelStyle):
    """Column-shard ``up_proj`` keeping a DTensor output (so ``chunk(2)`` splits the
    logical gate/up halves), row-shard ``down_proj``."""

    def _apply(self, module: nn.Module, device_mesh: DeviceMesh) -> nn.Module:
        return parallelize_module(
            module,
            device_mesh,
            {
                "up_proj": ColwiseParallel(output_layouts=Shard(-1), use_local_output=False),
                "down_proj": RowwiseParallel(input_layouts=Shard(-1)),
            },
        )


class MLAParallel(ParallelStyle):
    """Head-parallel MLA: the module records its head range and supplies the plan."""

    def _apply(self, module: nn.Module, device_mesh: DeviceMesh) -> nn.Module:
        module.shard_heads_over(device_mesh)  # type: ignore[operator]
        return parallelize_module(module, device_mesh, module.tensor_parallel_plan())  # type: ignore[operator]


def _vocab_style(module: nn.Module) -> ParallelStyle:
    if isinstance(module, nn.Embedding):
        return RowwiseParallel(input_layouts=Replicate())
    return ColwiseParallel(output_layouts=Replicate())


def _shard_style(module: nn.Module) -> ParallelStyle | None:
    shard = getattr(module, "shard", None)
    if hasattr(module, "tensor_parallel_style") and callable(module.tensor_parallel_style):
        return module.tensor_parallel_style() if shard else None
    if shard is None or not isinstance(module, (nn.Linear, nn.Embedding)):
        return None
    if shard == "colwise":
        return ColwiseParallel()
    if shard == "rowwise":
        return RowwiseParallel()
    if shard == "vocab":
        return _vocab_style(module)
    raise ValueError(f"Unknown shard style {shard!r} on {type(module).__name__}.")


def apply_tensor_parallel(model: nn.Module, mesh: DeviceMesh, *, mesh_dim: str = "tp") -> nn.Module:
    tp = mesh[mesh_dim]
    if tp.size() == 1:
        return model
    plan: dict[str, ParallelStyle] = {}
    covered: list[str] = []
    for name, sub in model.named_modules():
        if any(name.startswith(c + ".") for c in covered):
            continue
        style = _shard_style(sub)
        if style is not None:
            plan[name] = style
            if hasattr(sub, "tensor_parallel_style"):
                covered.append(name)
    if not plan:
        return model
    parallelize_module(model, tp, plan)
    for sub in model.modules():
        check = getattr(sub, "assert_tensor_parallel_compatible", None)
        if callable(check):
            check()
    log.info("Applied tensor parallel: %d sharded submodules.", len(plan))
    return model


class TensorParallel:
    """Strategy: place the model and shard it over the ``tp`` axis."""

    class Config(Fig["TensorParallel"]):
        mesh_dim: str = "tp"

    def __init__(self, config: Config | None = None) -> None:
        config = config or TensorParallel.Config()
        mesh = global_device_mesh()
        if mesh is None:
            raise RuntimeError("TensorParallel requires the MultiProcess runtime.")
        if mesh.mesh_dim_names is None or config.mesh_dim not in mesh.mesh_dim_names:
            raise ValueError(f"Mesh dimension {config.mesh_dim!r} not in {mesh.mesh_dim_names}.")
        self.device = torch.device("cuda", torch.cuda.current_device()) if mesh.device_type == "cuda" else torch.device(mesh.device_type)
        self.mesh = mesh
        self.mesh_dim = config.mesh_dim

    def __call__(self, model: nn.Module) -> nn.Module:
        return apply_tensor_parallel(place(model, self.device), self.mesh, mesh_dim=self.mesh_dim)
