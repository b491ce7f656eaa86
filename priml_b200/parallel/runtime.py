"""Process-global runtime: device resolution, process group and named mesh
(``priml/runtime.py:34-489``).

``MultiProcess`` binds ``LOCAL_RANK``, initializes ``torch.distributed``
(``nccl`` on CUDA, ``gloo`` on CPU, or ``"cpu:gloo,cuda:nccl"``), and builds a
named ``DeviceMesh`` over ``{"dp", "pp", "tp"}`` (one axis may be -1 and is
inferred; an ``"ep"`` axis is accepted for expert parallelism). Initialization
failures roll back what was acquired; the runtime only destroys a process group
it created itself.
"""

from __future__ import annotations

import datetime
import math
import os
from dataclasses import field
from typing import Any, Literal, Protocol

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh

from priml_b200.config import Fig

__all__ = [
    "MultiProcess",
    "RuntimeProtocol",
    "SingleProcess",
    "destroy_global_device_mesh",
    "get_device",
    "global_device_mesh",
    "initialize_global_device_mesh",
    "is_rank_zero",
    "runtime_initialized",
]


class RuntimeProtocol(Protocol):
    device: torch.device

    def initialize(self) -> None: ...

    def destroy(self) -> None: ...


def get_device(device: torch.device | str | None = "auto") -> torch.device:
    if device is None:
        return torch.get_default_device()
    if isinstance(device, str) and device == "auto":
        if torch.cuda.is_available():
            return torch.device("cuda")
        if torch.backends.mps.is_available():
            return torch.device("mps")
        return torch.device("cpu")
    return torch.device(device)


_mesh: DeviceMesh | None = None
_initialized = False
_owned_pg = False


def runtime_initialized() -> bool:
    return _initialized


def global_device_mesh() -> DeviceMesh | None:
    return _mesh


def is_rank_zero() -> bool:
    return not (dist.is_available() and dist.is_initialized()) or dist.get_rank() == 0


def _resolve_mesh_topology(topology: dict[str, int], world: int) -> dict[str, int]:
    sizes = dict(topology)
    unknown = [k for k, v in sizes.items() if v == -1]
    if len(unknown) > 1:
        raise ValueError(f"At most one mesh axis may be -1; got {topology}.")
    known = math.prod(v for v in sizes.values() if v != -1)
    if unknown:
        if world % known:
            raise ValueError(f"world size {world} not divisible by fixed mesh axes {topology}.")
        sizes[unknown[0]] = world // known
    if math.prod(sizes.values()) != world:
        raise ValueError(f"mesh {sizes} does not cover world size {world}.")
    return sizes


def initialize_global_device_mesh(
    *,
    device: torch.device,
    mesh_topology: dict[str, int],
    backend: str | None = None,
    timeout_s: float = 600.0,
) -> DeviceMesh:
    """Create (or adopt) the process group and the named global mesh."""
    global _mesh, _initialized, _owned_pg
    world = int(os.environ.get("WORLD_SIZE", "1"))
    sizes = _resolve_mesh_topology(mesh_topology, world)  # validate before acquiring anything
    if device.type == "cuda":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    created = False
    try:
        if not dist.is_initialized():
            be = backend or ("nccl" if device.type == "cuda" else "gloo")
            kwargs: dict[str, Any] = {"backend": be, "timeout": datetime.timedelta(seconds=timeout_s)}
            if device.type == "cuda" and be == "nccl":
                kwargs["device_id"] = device
            dist.init_process_group(**kwargs)
            created = True
        names = tuple(sizes)
        _mesh = init_device_mesh(device.type, tuple(sizes[n] for n in names), mesh_dim_names=names)
    except BaseException:
        if created and dist.is_initialized():
            dist.destroy_process_group()
        _mesh = None
        raise
    _owned_pg = created
    _initialized = True
    return _mesh


def destroy_global_device_mesh() -> None:
    global _mesh, _initialized, _owned_pg
    _mesh = None
    _initialized = False
    if _owned_pg and dist.is_initialized():
        dist.destroy_process_group()
    _owned_pg = False


class SingleProcess:
    """Non-distributed runtime (one GPU or CPU)."""

    class Config(Fig["SingleProcess"]):
        device: torch.device | str | None = "auto"
        deterministic: bool = False
        float32_matmul_precision: Literal["highest", "high", "medium"] | None = None

    def __init__(self, config: Config | None = None) -> None:
        config = config or SingleProcess.Config()
        self.config = config
        self.device = get_device(config.device)

    def initialize(self) -> None:
        global _initialized
        if self.config.deterministic:
            from priml_b200.math.seed import enable_determinism

            enable_determinism()
        if self.config.float32_matmul_precision is not None:
            torch.set_float32_matmul_precision(self.config.float32_matmul_precision)
        if self.device.type == "cuda" and self.device.index is not None:
            torch.cuda.set_device(self.device)
        _initialized = True

    def destroy(self) -> None:
        global _initialized
        _initialized = False


class MultiProcess:
    """One process per device under ``torchrun``; builds the global mesh."""

    class Config(Fig["MultiProcess"]):
        device: torch.device | str | None = "auto"
        deterministic: bool = False
        float32_matmul_precision: Literal["highest", "high", "medium"] | None = None
        backend: str | None = None
        mesh_topology: dict[str, int] = field(default_factory=lambda: {"dp": -1, "pp": 1, "tp": 1})
        timeout_s: float = 600.0

    def __init__(self, config: Config | None = None) -> None:
        config = config or MultiProcess.Config()
        self.config = config
        self.device = get_device(config.device)
        self.mesh: DeviceMesh | None = None

    def initialize(self) -> None:
        if self.config.deterministic:
            from priml_b200.math.seed import enable_determinism

            enable_determinism()
        if self.config.float32_matmul_precision is not None:
            torch.set_float32_matmul_precision(self.config.float32_matmul_precision)
        self.mesh = initialize_global_device_mesh(
            device=self.device,
            mesh_topology=self.config.mesh_topology,
            backend=self.config.backend,
            timeout_s=self.config.timeout_s,
        )
        if self.device.type == "cuda":
            self.device = torch.device("cuda", torch.cuda.current_device())

    def destroy(self) -> None:
        destroy_global_device_mesh()
