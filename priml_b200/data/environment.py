"""Batched environment protocol for on-policy RL (``priml/data/environment.py:35-100``)."""

from __future__ import annotations

from typing import Any, Protocol, runtime_checkable

from torch import Tensor

__all__ = ["BatchedEnvironmentProtocol", "EnvironmentStep"]


class EnvironmentStep(Protocol):
    """One transition of every worker: next observations (post-reset where ``done``),
    rewards ``[envs]``, terminal flags ``[envs]`` and diagnostics ``info``."""

    observation: Tensor
    reward: Tensor
    done: Tensor
    info: dict[str, Tensor]


@runtime_checkable
class BatchedEnvironmentProtocol(Protocol):
    """An auto-resetting batch of environments with a discrete action space."""

    num_actions: int
    observation_size: int
    reward_ceiling: float

    def reset(self, num_envs: int) -> Tensor: ...

    def step(self, actions: Tensor) -> EnvironmentStep: ...

    def state_dict(self) -> dict[str, Any]: ...

    def load_state_dict(self, state_dict: dict[str, Any]) -> None: ...
