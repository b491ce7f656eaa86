"""Structural types of the training layer (``priml/train/custom_types.py:47-365``).

Anything that satisfies these protocols plugs into :class:`TrainStep` /
:class:`TrainLoop`: checkpointable objects (``state_dict`` /
``load_state_dict``), optimizers, EMAs, checkpointers, trackers, profilers and
phase timers.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator, Mapping
from contextlib import AbstractContextManager
from typing import Any, Protocol, TypedDict, overload, runtime_checkable

import torch
from torch import Tensor, nn

__all__ = [
    "CheckpointableProtocol",
    "CheckpointingProtocol",
    "CudaEventProtocol",
    "EMAProtocol",
    "ModelOutput",
    "ModuleLike",
    "OptimizerProtocol",
    "PhaseTimerProtocol",
    "ProfileProtocol",
    "TrackerProtocol",
    "TrainStepOutput",
]


@runtime_checkable
class ModelOutput(Protocol):
    """A tensor or a mapping of tensors returned by a model."""

    def __getitem__(self, key: Any) -> Any: ...


class TrainStepOutput(TypedDict, total=False):
    loss: Tensor
    """Per-sample (unreduced) loss."""
    model: Any
    num_samples: int
    stepped: bool


@runtime_checkable
class CheckpointableProtocol(Protocol):
    def state_dict(self) -> Mapping[str, Any]: ...

    def load_state_dict(self, state_dict: Mapping[str, Any]) -> Any: ...


@runtime_checkable
class OptimizerProtocol(CheckpointableProtocol, Protocol):
    param_groups: list[dict[str, Any]]

    @overload
    def step(self, closure: None = None) -> None: ...
    @overload
    def step(self, closure: Callable[[], Tensor | float]) -> Tensor | float: ...
    def step(self, closure: Callable[[], Tensor | float] | None = None) -> Tensor | float | None: ...

    def zero_grad(self, set_to_none: bool = False) -> None: ...


@runtime_checkable
class ModuleLike(CheckpointableProtocol, Protocol):
    def parameters(self) -> Iterator[nn.Parameter]: ...

    def buffers(self) -> Iterator[Tensor]: ...

    def to(self, device: torch.device | str | None = None) -> Any: ...

    def eval(self) -> Any: ...

    def train(self, mode: bool = True) -> Any: ...

    def requires_grad_(self, requires_grad: bool = True) -> Any: ...


@runtime_checkable
class EMAProtocol(CheckpointableProtocol, Protocol):
    def __call__(self, model: Any) -> None: ...

    def apply_to(self, model: nn.Module) -> AbstractContextManager[None]: ...


@runtime_checkable
class CheckpointingProtocol(Protocol):
    def maybe_save(self, target: CheckpointableProtocol, step: int) -> bool: ...

    def save(self, target: CheckpointableProtocol, step: int) -> Any: ...

    def load(self, target: CheckpointableProtocol, max_steps: float = ..., guard: bool = ...) -> int | None: ...


@runtime_checkable
class TrackerProtocol(Protocol):
    def log_metrics(self, metrics: Mapping[str, float], step: int) -> None: ...

    def close(self) -> None: ...


@runtime_checkable
class ProfileProtocol(Protocol):
    def on_step_start(self, step: int) -> None: ...

    def on_step_end(self, step: int) -> None: ...

    def cleanup(self) -> None: ...


@runtime_checkable
class CudaEventProtocol(Protocol):
    def record(self) -> None: ...

    def synchronize(self) -> None: ...

    def elapsed_time(self, end_event: Any) -> float: ...


@runtime_checkable
class PhaseTimerProtocol(Protocol):
    @property
    def cuda_events_enabled(self) -> bool: ...

    def phase(self, name: str) -> AbstractContextManager[None]: ...


@runtime_checkable
class ParallelStrategyProtocol(Protocol):
    """A parallel strategy: ``__call__`` places, shards and materializes a model on ``device``."""

    device: torch.device

    def __call__(self, model: nn.Module) -> nn.Module: ...


class ModelQuantizationProtocol(Protocol):
    """A model quantization: ``__call__`` returns the model with its layers converted."""

    def __call__(self, model: nn.Module) -> nn.Module: ...
