"""The learner's view of Craftax: batched reset / step with auto-restart (``priml/baselines/craftax/env.py``).

Implements :class:`priml_b200.data.environment.BatchedEnvironmentProtocol`. The
environment owns its generator, so the worlds do not depend on how many actions
the policy sampled. Finished workers restart in freshly generated worlds; like
the reference (optimistic resets) only ``num_envs / optimistic_reset_ratio``
worlds are generated per step in which any worker finished, dealt to the
finished workers in turn.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import Tensor

from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game import observation, world
from priml_b200.baselines.craftax.game import step as rules
from priml_b200.baselines.craftax.game.state import GameState
from priml_b200.config import Fig
from priml_b200.parallel.runtime import get_device

__all__ = ["CraftaxEnv", "CraftaxStep"]


@dataclass(frozen=True, slots=True, kw_only=True)
class CraftaxStep:
    observation: Tensor
    reward: Tensor
    done: Tensor
    info: dict[str, Tensor]


class CraftaxEnv:
    class Config(Fig["CraftaxEnv"]):
        num_envs: int = 256
        device: str = "auto"
        seed: int = 0
        view: tuple[int, int] = C.OBS_DIM
        optimistic_reset_ratio: int = 16

    def __init__(self, config: Config) -> None:
        if config.num_envs <= 0 or config.optimistic_reset_ratio <= 0 or min(config.view) <= 0:
            raise ValueError("num_envs, optimistic_reset_ratio and view must be positive")
        self.config = config
        self.num_actions = len(C.Action)
        self.observation_size = observation.observation_size(config.view)
        self.reward_ceiling = C.REWARD_CEILING
        self.device = get_device(config.device)
        self._num_envs = config.num_envs
        self._generator = torch.Generator(device=self.device)
        self._generator.manual_seed(config.seed)
        self._state: GameState | None = None

    @property
    def state(self) -> GameState:
        if self._state is None:
            raise RuntimeError("reset the environment before reading it")
        return self._state

    def reset(self, num_envs: int = 0) -> Tensor:
        if num_envs:
            self._num_envs = num_envs
        self._state = world.generate(self._num_envs, generator=self._generator, device=self.device)
        return observation.render(self._state, self.config.view)

    def step(self, actions: Tensor) -> CraftaxStep:
        s, reward = rules.step(self.state, actions.to(self.device), generator=self._generator)
        done = rules.is_done(s)
        unlocked = s.achievements & done[:, None]
        pct = unlocked.float() * 100.0  # one kernel; the entries are column views
        info = {f"Achievements/{a.name.lower()}": pct[:, int(a)] for a in C.Achievement}
        if bool(done.any()):
            pool = max(1, s.num_envs // self.config.optimistic_reset_ratio)
            want = min(int(done.sum()), pool)
            fresh = world.generate(want, generator=self._generator, device=self.device)
            if want < s.num_envs:
                rank = done.long().cumsum(0) - 1
                fresh = fresh.take(rank.clamp(min=0) % want)
            s = s.select(done, fresh)
        self._state = s
        return CraftaxStep(observation=observation.render(s, self.config.view), reward=reward, done=done, info=info)

    def state_dict(self) -> dict[str, Any]:
        return {"generator": self._generator.get_state(), "num_envs": self._num_envs,
                "state": {} if self._state is None else self._state.state_dict()}  # fmt: skip

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self._generator.set_state(s["generator"])
        self._num_envs = int(s["num_envs"])
        if not s["state"]:
            self._state = None
            return
        if self._state is None:
            self.reset()
        self.state.load_state_dict(s["state"])
