"""Seeding and RNG state capture (``priml/math/seed.py:34-410``).

``salt(*args)`` derives a 31-bit integer from stable-repr primitives (the MD5
of their tuple repr, masked to 31 bits -- the same rule as the reference so
salted seeds agree). ``set_seed_distributed`` broadcasts rank 0's base seed and
salts it locally per mesh axis; RNG state round-trips python/numpy/torch/cuda
plus device identities.
"""

from __future__ import annotations

import hashlib
import os
import random
import secrets
import warnings
from typing import Any, TypedDict

import numpy as np
import torch
import torch.distributed as dist

__all__ = [
    "RngState",
    "dataloader_worker_init_fn",
    "enable_determinism",
    "get_rng_state",
    "make_seed",
    "salt",
    "set_rng_state",
    "set_seed_distributed",
    "set_seed_local",
]

_STABLE = (str, bytes, int, float, bool, type(None))
_numpy_rng = np.random.default_rng()


class RngState(TypedDict, total=False):
    python: Any
    torch: torch.Tensor
    numpy: Any
    cuda: list[torch.Tensor]
    cuda_uuids: list[str]


def enable_determinism(*, cudnn: bool = True, sdpa: bool = True) -> None:
    """Deterministic algorithms (and cuDNN / math-SDPA) for reproducibility runs."""
    os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")
    torch.use_deterministic_algorithms(True, warn_only=True)
    if cudnn:
        torch.backends.cudnn.deterministic = True
        torch.backends.cudnn.benchmark = False
    if sdpa and torch.cuda.is_available():
        torch.backends.cuda.enable_flash_sdp(False)
        torch.backends.cuda.enable_mem_efficient_sdp(False)
        torch.backends.cuda.enable_math_sdp(True)


def salt(*args: object) -> int:
    for a in args:
        if not isinstance(a, _STABLE):
            raise TypeError(f"salt() requires primitive args with stable repr; got {type(a).__name__}.")
    return int(hashlib.md5(str(args).encode()).hexdigest(), 16) & 0x7FFFFFFF  # noqa: S324


def make_seed() -> int:
    return secrets.randbits(63) or 1


def set_seed_local(seed: int | None = None) -> int:
    """Seed python, numpy and torch (all devices); returns the seed used."""
    global _numpy_rng
    if seed is None:
        seed = make_seed()
    random.seed(seed)
    np.random.seed(seed % (2**32))
    _numpy_rng = np.random.default_rng(seed)
    torch.manual_seed(seed)
    return seed


def dataloader_worker_init_fn(worker_id: int) -> None:
    base = torch.initial_seed()
    s = (base + salt("worker", worker_id)) % (2**63)
    random.seed(s)
    np.random.seed(s % (2**32))


def set_seed_distributed(seed: int | None = None, *, group: Any = None, axis_salts: tuple[object, ...] = ()) -> int:
    """Rank 0's seed (or ``seed``) broadcast to all ranks, then salted locally
    by ``axis_salts`` (e.g. this rank's coordinate on a mesh axis)."""
    if seed is None:
        seed = make_seed()
    if dist.is_available() and dist.is_initialized():
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")
        t = torch.tensor([seed], dtype=torch.int64, device=dev)
        src = 0 if group is None else dist.get_global_rank(group, 0)
        dist.broadcast(t, src=src, group=group)
        seed = int(t.item())
    if axis_salts:
        seed = (seed + salt(*axis_salts)) % (2**63) or 1
    return set_seed_local(seed)


def _device_identity(i: int) -> str:
    try:
        props = torch.cuda.get_device_properties(i)
        return str(getattr(props, "uuid", "")) or f"{props.name}:{getattr(props, 'pci_bus_id', i)}"
    except Exception:  # noqa: BLE001
        return f"cuda:{i}"


def get_rng_state() -> RngState:
    state: RngState = {
        "python": random.getstate(),
        "torch": torch.get_rng_state(),
        "numpy": _numpy_rng.bit_generator.state,
    }
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        state["cuda"] = torch.cuda.get_rng_state_all()
        state["cuda_uuids"] = [_device_identity(i) for i in range(torch.cuda.device_count())]
    return state


def set_rng_state(state: RngState) -> None:
    random.setstate(state["python"])
    torch.set_rng_state(state["torch"].cpu() if isinstance(state["torch"], torch.Tensor) else state["torch"])
    if "numpy" in state:
        _numpy_rng.bit_generator.state = state["numpy"]
    if "cuda" in state and torch.cuda.is_available():
        saved = state.get("cuda_uuids")
        if saved is not None:
            now = [_device_identity(i) for i in range(torch.cuda.device_count())]
            if now[: len(saved)] != saved:
                warnings.warn("CUDA devices differ from the checkpoint's; restoring RNG by index.", stacklevel=2)
        torch.cuda.set_rng_state_all([s.cpu() for s in state["cuda"]][: torch.cuda.device_count()])
