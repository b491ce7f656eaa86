"""Model placement / sharding strategies (``priml/train/parallelism.py:34-526``).

* ``NoParallel``           materialize (meta) or move the model.
* ``DataParallel``         DDP via ``replicate`` over the ``dp`` mesh axis.
* ``FullySharded``         FSDP2 ``fully_shard`` over ``dp`` with a mixed-precision policy.
* ``HybridSharded``        HSDP: replicate over one axis, shard over the other.
* ``RecursiveFullySharded`` per-block ``fully_shard`` (leaves first), root last.

Meta materialization (``materialize_meta``) allocates on the target device,
NaN-poisons, calls the model's ``reset_parameters`` and audits for NaNs left
behind -- a model whose containers forget to recurse fails loudly.

These strategies drive NCCL through ``torch.distributed``; the fused
all-gather-GEMM / reduce-scatter-optimizer path lives in
:mod:`priml_b200.parallel.fsdp`.
"""

from __future__ import annotations

from collections.abc import Sequence

from dataclasses import field
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from priml_b200.config import Fig
from priml_b200.parallel.runtime import get_device, global_device_mesh

__all__ = [
    "DataParallel",
    "FullySharded",
    "HybridSharded",
    "NoParallel",
    "RecursiveFullySharded",
    "RecursiveSharded",
    "materialize_meta",
    "place",
]

_DTYPES = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}


def _dtype(x: Any) -> torch.dtype | None:
    if x is None or isinstance(x, torch.dtype):
        return x
    return _DTYPES[str(x)]


def _has_meta(model: nn.Module) -> bool:
    return any(t.is_meta for t in (*model.parameters(), *model.buffers()))


def materialize_meta(model: nn.Module, device: torch.device) -> nn.Module:
    """Allocate meta storage on ``device``, poison with NaN, re-initialize, audit."""
    model.to_empty(device=device)
    with torch.no_grad():
        for t in (*model.parameters(), *model.buffers()):
            local = t._local_tensor if hasattr(t, "_local_tensor") else t  # noqa: SLF001
            if local.is_floating_point():
                local.fill_(float("nan"))
    if not hasattr(model, "reset_parameters"):
        raise RuntimeError(f"{type(model).__name__} has no reset_parameters(); cannot materialize from meta.")
    model.reset_parameters()  # type: ignore[operator]
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    bad = []
    for name, t in (*model.named_parameters(), *model.named_buffers()):
        local = t._local_tensor if hasattr(t, "_local_tensor") else t  # noqa: SLF001
        if local.is_floating_point() and local.numel() and bool(torch.isnan(local).any()):
            bad.append(name)
    if bad:
        raise RuntimeError(f"reset_parameters() left NaN (uninitialized) tensors: {bad[:8]}")
    return model


def place(model: nn.Module, device: torch.device) -> nn.Module:
    return materialize_meta(model, device) if _has_meta(model) else model.to(device)


def _mesh_axis(name: str) -> Any:
    mesh = global_device_mesh()
    if mesh is None:
        return None
    return mesh[name] if name in (mesh.mesh_dim_names or ()) else None


class NoParallel:
    class Config(Fig["NoParallel"]):
        device: torch.device | str | None = "auto"

    def __init__(self, config: Config | None = None) -> None:
        config = config or NoParallel.Config()
        self.device = get_device(config.device)

    def __call__(self, model: nn.Module) -> nn.Module:
        return place(model, self.device)


class DataParallel:
    """DDP (gradient all-reduce in buckets) over the ``dp`` axis."""

    class Config(Fig["DataParallel"]):
        device: torch.device | str | None = "auto"
        mesh_dim: str = "dp"
        bucket_cap_mb: int = 25
        find_unused_parameters: bool = False
        gradient_as_bucket_view: bool = True

    def __init__(self, config: Config | None = None) -> None:
        self.config = config or DataParallel.Config()
        self.device = get_device(self.config.device)

    def __call__(self, model: nn.Module) -> nn.Module:
        model = place(model, self._device())
        from torch.distributed._composable.replicate import replicate

        mesh = _mesh_axis(self.config.mesh_dim)
        kwargs: dict[str, Any] = {
            "bucket_cap_mb": self.config.bucket_cap_mb,
            "find_unused_parameters": self.config.find_unused_parameters,
            "gradient_as_bucket_view": self.config.gradient_as_bucket_view,
        }
        if mesh is not None:
            kwargs["device_mesh"] = mesh
        replicate(model, **kwargs)
        return model

    def _device(self) -> torch.device:
        if self.device.type == "cuda" and torch.cuda.is_available():
            return torch.device("cuda", torch.cuda.current_device())
        return self.device


class FullySharded:
    """FSDP2 over ``mesh_dim``; optionally one ``fully_shard`` per transformer block."""

    class Config(Fig["FullySharded"]):
        device: torch.device | str | None = "auto"
        mesh_dim: str = "dp"
        mp_param_dtype: Any = None
        mp_reduce_dtype: Any = None
        mp_output_dtype: Any = None
        reshard_after_forward: bool = True
        per_block: bool = True
        """Shard each ``blocks[i]`` separately (prefetchable units) before the root."""

    def __init__(self, config: Config | None = None) -> None:
        self.config = config or FullySharded.Config()
        self.device = get_device(self.config.device)

    def _policy(self) -> Any:
        from torch.distributed.fsdp import MixedPrecisionPolicy

        c = self.config
        return MixedPrecisionPolicy(
            param_dtype=_dtype(c.mp_param_dtype),
            reduce_dtype=_dtype(c.mp_reduce_dtype),
            output_dtype=_dtype(c.mp_output_dtype),
        )

    def _mesh(self) -> Any:
        return _mesh_axis(self.config.mesh_dim)

    def __call__(self, model: nn.Module) -> nn.Module:
        from torch.distributed.fsdp import fully_shard

        meta = _has_meta(model)
        mesh = self._mesh()
        policy = self._policy()
        if self.config.per_block:
            blocks = getattr(model, "blocks", None)
            if isinstance(blocks, nn.ModuleList):
                for blk in blocks:
                    fully_shard(blk, mesh=mesh, mp_policy=policy, reshard_after_forward=self.config.reshard_after_forward)
        fully_shard(model, mesh=mesh, mp_policy=policy, reshard_after_forward=False)
        dev = torch.device("cuda", torch.cuda.current_device()) if self.device.type == "cuda" else self.device
        if meta:
            materialize_meta(model, dev)
        else:
            model.to(dev)
        return model


class HybridSharded(FullySharded):
    """HSDP: replicate over ``replicate_dim``, shard over ``shard_dim``."""

    class Config(Fig["HybridSharded"]):
        device: torch.device | str | None = "auto"
        replicate_dim: str = "dp"
        shard_dim: str = "tp"
        mp_param_dtype: Any = None
        mp_reduce_dtype: Any = None
        mp_output_dtype: Any = None
        reshard_after_forward: bool = True
        per_block: bool = True

    def _mesh(self) -> Any:
        mesh = global_device_mesh()
        if mesh is None:
            return None
        return mesh[(self.config.replicate_dim, self.config.shard_dim)]  # type: ignore[attr-defined]


class RecursiveFullySharded(FullySharded):
    """``fully_shard`` every module whose class name is in ``block_types`` (leaves
    first; BatchNorm kept in fp32 as its own unit), then the root."""

    class Config(Fig["RecursiveFullySharded"]):
        device: torch.device | str | None = "auto"
        mesh_dim: str = "dp"
        block_types: list[str] = field(default_factory=lambda: ["TransformerBlock"])
        mp_param_dtype: Any = None
        mp_reduce_dtype: Any = None
        mp_output_dtype: Any = None
        reshard_after_forward: bool = True
        per_block: bool = False

    def __call__(self, model: nn.Module) -> nn.Module:
        from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

        meta = _has_meta(model)
        mesh, policy = self._mesh(), self._policy()
        mods = [m for m in model.modules() if type(m).__name__ in self.config.block_types and m is not model]
        for m in reversed(mods):
            fully_shard(m, mesh=mesh, mp_policy=policy, reshard_after_forward=self.config.reshard_after_forward)
        for m in model.modules():
            if isinstance(m, nn.modules.batchnorm._BatchNorm):  # noqa: SLF001
                fully_shard(m, mesh=mesh, mp_policy=MixedPrecisionPolicy(param_dtype=torch.float32))
        fully_shard(model, mesh=mesh, mp_policy=policy, reshard_after_forward=False)
        dev = torch.device("cuda", torch.cuda.current_device()) if self.device.type == "cuda" else self.device
        if meta:
            materialize_meta(model, dev)
        else:
            model.to(dev)
        return model


class RecursiveSharded(RecursiveFullySharded):
    """The reference's name and configuration for recursive FSDP (``priml/train/parallelism.py:275-330``):
    modules are selected by class (``module_types``) instead of by class name; sharding, mixed
    precision and materialization are :class:`RecursiveFullySharded`'s."""

    class Config(Fig["RecursiveSharded"]):
        device: torch.device | str | None = "auto"
        mesh_dim: str = "dp"
        module_types: Sequence[type[nn.Module]] = ()
        reshard_after_forward: bool = True
        mp_param_dtype: Any = None
        mp_reduce_dtype: Any = None
        mp_output_dtype: Any = None
        per_block: bool = False

        @property
        def block_types(self) -> list[str]:
            return [t.__name__ for t in self.module_types]
