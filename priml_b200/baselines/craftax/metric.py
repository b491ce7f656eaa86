"""Craftax evaluation: normalized return and the Crafter score (``priml/baselines/craftax/metric.py``).

``update(_, policy=...)`` plays the given policy (sampling its softmax) in fresh
evaluation worlds for ``steps`` steps on ``num_envs`` workers and records every
finished episode's return, length and achievements. ``compute()`` reports the
mean return as a percentage of the 226-point ceiling and the Crafter score
(Hafner 2021): the geometric mean over achievements of the success rates in
percent, ``exp(mean(ln(1 + s_i))) - 1``.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import Tensor

from priml_b200.baselines.craftax.env import CraftaxEnv
from priml_b200.baselines.craftax.game import constants as C
from priml_b200.config import Fig

__all__ = ["CraftaxScore", "crafter_score_pct"]


def crafter_score_pct(success_pct: list[float]) -> float:
    return math.exp(sum(math.log(1.0 + s) for s in success_pct) / len(success_pct)) - 1.0


class CraftaxScore:
    class Config(Fig["CraftaxScore"]):
        num_envs: int = 64
        steps: int = 10_000
        seed: int = 42
        view: tuple[int, int] = C.OBS_DIM
        device: str = "auto"

    def __init__(self, config: Config | None = None) -> None:
        self.config = config or CraftaxScore.Config()
        if self.config.num_envs <= 0 or self.config.steps <= 0:
            raise ValueError("evaluation geometry must be positive")
        self.reset()

    def reset(self) -> None:
        self._returns: list[float] = []
        self._lengths: list[int] = []
        self._unlocked: list[list[bool]] = []

    def update(self, logits: Tensor | None = None, **batch: Any) -> None:
        del logits
        policy = batch.get("policy")
        if policy is not None:
            self.play(policy)

    @torch.no_grad()
    def play(self, policy: Any) -> None:
        c = self.config
        env = CraftaxEnv.Config(num_envs=c.num_envs, device=c.device, seed=c.seed, view=c.view).make()
        obs = env.reset()
        g = torch.Generator(device=obs.device)
        g.manual_seed(c.seed)
        ret = torch.zeros(c.num_envs, device=obs.device)
        length = torch.zeros(c.num_envs, dtype=torch.long, device=obs.device)
        for _ in range(c.steps):
            out = policy(obs)
            logits = out[0] if isinstance(out, tuple) else out
            a = torch.multinomial(logits.float().softmax(-1), 1, generator=g)[:, 0]
            ach_before = env.state.achievements.clone()
            t = env.step(a)
            ret += t.reward
            length += 1
            if bool(t.done.any()):
                d = t.done
                self._returns += ret[d].tolist()
                self._lengths += length[d].tolist()
                self._unlocked += ach_before[d].tolist()
                ret, length = ret * ~d, length * ~d
            obs = t.observation

    def compute(self) -> dict[str, float]:
        if not self._returns:
            return {"episodes": 0.0}
        n = len(self._returns)
        rates = [100.0 * sum(row[i] for row in self._unlocked) / n for i in range(C.NUM_ACHIEVEMENTS)]
        mean = sum(self._returns) / n
        return {"normalized_return_pct": mean / C.REWARD_CEILING * 100.0, "score_pct": crafter_score_pct(rates),
                "mean_return": mean, "achievements_pct": sum(rates) / len(rates), "episodes": float(n),
                "episode_length": sum(self._lengths) / n}  # fmt: skip

    def state_dict(self) -> dict[str, Any]:
        return {"returns": list(self._returns), "lengths": list(self._lengths), "unlocked": [list(r) for r in self._unlocked]}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self._returns, self._lengths = list(s["returns"]), list(s["lengths"])
        self._unlocked = [list(r) for r in s["unlocked"]]
