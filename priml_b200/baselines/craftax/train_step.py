"""On-policy learners for Craftax (``priml/baselines/craftax/train_step.py``,
``rnn_train_step.py``, ``pqn_train_step.py``).

Each ``train_step()`` call is one update: collect ``rollout_steps`` steps from
every worker (the environment generates its own data; the loop's batch is
ignored), then optimize. Shared by the three learners: Adam (RAdam for PQN) with
the rate annealed linearly to zero over ``total_train_steps``, a global
gradient-norm clip, episode bookkeeping (return, length, normalized return =
return / 226 x 100) and checkpointable environment / generator state.

* :class:`CraftaxTrainStep` -- PPO with GAE: clipped ratio objective, clipped
  value loss, entropy bonus, advantages normalized per minibatch, ``num_epochs``
  passes of ``num_minibatches`` shuffled minibatches.
* :class:`CraftaxRNNTrainStep` -- the same objective on a GRU policy; the
  recurrent state is carried across updates and minibatches are whole worker
  sequences replayed from the rollout's initial state.
* :class:`CraftaxGTrXLTrainStep` -- the recurrent objective on a gated
  Transformer-XL whose state is a per-layer memory of the last 128 inputs.
* :class:`CraftaxPQNTrainStep` -- PQN (Gallici et al. 2024): epsilon-greedy
  rollouts from a recurrent Q-network, Peng's Q(lambda) targets from the
  rollout's own Q-values, squared error on the chosen actions' Q-values.
"""

from __future__ import annotations

from dataclasses import field
from typing import Any

import torch
from torch import Tensor
from torch.nn import functional as F

from priml_b200.baselines.craftax.env import CraftaxEnv
from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game.observation import observation_size
from priml_b200.baselines.craftax.model import (
    ActorCritic,
    ActorCriticGTrXL,
    ActorCriticRNN,
    RecurrentQNetwork,
    epsilon_at,
)
from priml_b200.config import Makes, PartialConfig
from priml_b200.math.advantage import explained_variance, generalized_advantage, q_lambda_targets
from priml_b200.train.train_step import TrainStep, TrainStepOutput

__all__ = ["CraftaxGTrXLTrainStep", "CraftaxPQNTrainStep", "CraftaxRNNTrainStep", "CraftaxTrainStep", "ppo_terms"]


def ppo_terms(logits: Tensor, actions: Tensor, old_log_prob: Tensor, value: Tensor, old_value: Tensor,
              advantage: Tensor, target: Tensor, clip: float) -> dict[str, Tensor]:  # fmt: skip
    """Clipped surrogate, clipped value regression, entropy and diagnostics (advantages normalized here)."""
    log_probs = logits.float().log_softmax(-1)
    chosen = log_probs.gather(-1, actions[..., None].long())[..., 0]
    adv = (advantage - advantage.mean()) / (advantage.std() + 1e-8)
    log_ratio = chosen - old_log_prob
    ratio = log_ratio.exp()
    policy = -torch.minimum(ratio * adv, ratio.clamp(1 - clip, 1 + clip) * adv).mean()
    value = value.float()
    clipped = old_value + (value - old_value).clamp(-clip, clip)
    value_loss = 0.5 * torch.maximum((value - target) ** 2, (clipped - target) ** 2).mean()
    entropy = -(log_probs.exp() * log_probs).sum(-1).mean()
    return {"policy": policy, "value": value_loss, "entropy": entropy,
            "approx_kl": ((ratio - 1) - log_ratio).mean().detach(),
            "clip_fraction": ((ratio - 1).abs() > clip).float().mean().detach()}  # fmt: skip


class _RolloutStep(TrainStep):
    class Config(TrainStep.Config, kw_only=False):
        env: Any = field(default_factory=CraftaxEnv.Config)
        rollout_steps: int = 16
        num_epochs: int = 4
        num_minibatches: int = 8
        learning_rate: float = 3e-4
        anneal_learning_rate: bool = True
        total_train_steps: int = 244
        discount: float = 0.99
        trace_decay: float = 0.8
        max_grad_norm: float = 1.0
        seed: int = 0
        dtype_autocast: torch.dtype | None = torch.bfloat16

        def finalize(self):  # noqa: ANN201
            self.model.observation_size = observation_size(self.env.view)
            self.model.num_actions = len(C.Action)
            self.optimizer = self._optimizer()
            return super().finalize()

        def _optimizer(self) -> Any:
            return PartialConfig(torch.optim.Adam, lr=self.learning_rate, eps=1e-5)

    def __init__(self, config: Config) -> None:
        if min(config.rollout_steps, config.num_epochs, config.num_minibatches, config.total_train_steps) <= 0:
            raise ValueError("rollout geometry and total_train_steps must be positive")
        if not (0.0 <= config.discount <= 1.0 and 0.0 <= config.trace_decay <= 1.0):
            raise ValueError("discount and trace_decay must lie in [0, 1]")
        rng = torch.get_rng_state()
        torch.manual_seed(config.seed)
        try:
            super().__init__(config)
        finally:
            torch.set_rng_state(rng)
        self.config = config
        self.env = config.env.make()
        self._generator = torch.Generator(device=self.device)
        self._generator.manual_seed(config.seed)
        self._observation = self.env.reset().to(self.device)
        n = self._observation.shape[0]
        if n % config.num_minibatches and isinstance(self, (CraftaxRNNTrainStep, CraftaxPQNTrainStep)):
            raise ValueError("recurrent minibatches split the workers: num_minibatches must divide num_envs")
        self._done = torch.zeros(n, dtype=torch.bool, device=self.device)
        self._ep_return = torch.zeros(n, device=self.device)
        self._ep_length = torch.zeros(n, dtype=torch.long, device=self.device)
        self._finished = torch.zeros(3, dtype=torch.float64, device=self.device)  # episodes, return sum, length sum

    @property
    def global_step(self) -> int:
        return self.timer_step.global_count

    @property
    def steps_per_update(self) -> int:
        return int(self._observation.shape[0]) * self.config.rollout_steps

    def preprocess_batch(self, batch: dict[str, Any]) -> dict[str, Any]:
        return batch

    def on_epoch_end(self) -> None:
        """Updates are self-contained; nothing to flush at an epoch boundary."""

    def _lr(self) -> None:
        scale = max(0.0, 1.0 - self.global_step / self.config.total_train_steps) if self.config.anneal_learning_rate else 1.0
        for g in self.optimizer.param_groups:
            g["lr"] = self.config.learning_rate * scale

    def _record(self, reward: Tensor, done: Tensor) -> None:
        """Sums over finished episodes stay on the device (no host read per environment step)."""
        self._ep_return += reward
        self._ep_length += 1
        d = done.to(torch.float64)
        self._finished += torch.stack([d.sum(), (self._ep_return * d).sum(), (self._ep_length * d).sum()])
        self._ep_return = self._ep_return * ~done
        self._ep_length = self._ep_length * ~done

    def _episode_metrics(self) -> dict[str, float]:
        n, ret_sum, len_sum = self._finished.tolist()
        self._finished.zero_()
        if n == 0:
            return {"episodes": 0.0}
        ret = ret_sum / n
        return {"episodes": n, "episode_return": ret, "episode_length": len_sum / n,
                "normalized_return_pct": ret / C.REWARD_CEILING * 100.0}  # fmt: skip

    def _apply(self, loss: Tensor) -> Tensor:
        self.optimizer.zero_grad(set_to_none=True)
        loss.backward()
        norm = torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.config.max_grad_norm)
        self.optimizer.step()
        return norm

    def train_step(self, **batch: Any) -> TrainStepOutput:
        del batch
        self.model.train()
        rollout = self.collect()
        self._lr()
        with self.timer_step:
            metrics = self.optimize(rollout)
        metrics.update(self._episode_metrics())
        loss = metrics.pop("loss")
        return TrainStepOutput(loss=loss.reshape(1), metrics=metrics, stepped=True, num_samples=self.steps_per_update)

    def train_loss(self, **batch: Any) -> TrainStepOutput:
        del batch
        with torch.no_grad():
            return TrainStepOutput(loss=self.evaluate_loss(self.collect()).reshape(1))

    def eval_loss(self, **batch: Any) -> TrainStepOutput:
        was = self.model.training
        self.model.eval()
        try:
            return self.train_loss(**batch)
        finally:
            self.model.train(was)

    def state_dict(self) -> dict[str, Any]:
        return super().state_dict() | {"env": self.env.state_dict(), "generator": self._generator.get_state(),
                                        "observation": self._observation, "done": self._done,
                                        "episode_return": self._ep_return, "episode_length": self._ep_length}  # fmt: skip

    def load_state_dict(self, s: dict[str, Any]) -> None:
        super().load_state_dict(s)
        self.env.load_state_dict(s["env"])
        self._generator.set_state(s["generator"])
        self._observation, self._done = s["observation"], s["done"]
        self._ep_return, self._ep_length = s["episode_return"], s["episode_length"]

    # subclasses
    def collect(self) -> dict[str, Tensor]:
        raise NotImplementedError

    def optimize(self, rollout: dict[str, Tensor]) -> dict[str, Any]:
        raise NotImplementedError

    def evaluate_loss(self, rollout: dict[str, Tensor]) -> Tensor:
        raise NotImplementedError


class CraftaxTrainStep(_RolloutStep):
    """PPO on the feed-forward actor-critic."""

    class Config(Makes["CraftaxTrainStep"], _RolloutStep.Config, kw_only=False):
        model: Any = field(default_factory=ActorCritic.Config)
        clip_epsilon: float = 0.2
        entropy_coefficient: float = 0.01
        value_coefficient: float = 0.5

    @torch.no_grad()
    def collect(self) -> dict[str, Tensor]:
        obs, act, logp, val, rew, done = [], [], [], [], [], []
        for _ in range(self.config.rollout_steps):
            with self._autocast():
                logits, value = self.model(self._observation)
            lp = logits.float().log_softmax(-1)
            a = torch.multinomial(lp.exp(), 1, generator=self._generator)[:, 0]
            obs.append(self._observation)
            act.append(a)
            logp.append(lp.gather(-1, a[:, None])[:, 0])
            val.append(value.float())
            t = self.env.step(a)
            self._observation = t.observation
            rew.append(t.reward)
            done.append(t.done)
            self._record(t.reward, t.done)
        with self._autocast():
            _, last = self.model(self._observation)
        value = torch.stack(val)
        adv, target = generalized_advantage(rewards=torch.stack(rew), values=value, dones=torch.stack(done),
                                            last_value=last.float(), discount=self.config.discount,
                                            trace_decay=self.config.trace_decay)  # fmt: skip
        return {"observation": torch.stack(obs), "action": torch.stack(act), "log_prob": torch.stack(logp),
                "value": value, "advantage": adv, "target": target}  # fmt: skip

    def _loss(self, mb: dict[str, Tensor]) -> tuple[Tensor, dict[str, Tensor]]:
        with self._autocast():
            logits, value = self.model(mb["observation"])
        c = self.config
        t = ppo_terms(logits, mb["action"], mb["log_prob"], value, mb["value"], mb["advantage"], mb["target"],
                      c.clip_epsilon)  # fmt: skip
        return t["policy"] + c.value_coefficient * t["value"] - c.entropy_coefficient * t["entropy"], t

    def optimize(self, rollout: dict[str, Tensor]) -> dict[str, Any]:
        flat = {k: v.flatten(0, 1) for k, v in rollout.items()}
        n = flat["action"].shape[0]
        out: dict[str, Any] = {}
        for _ in range(self.config.num_epochs):
            order = torch.randperm(n, device=self.device, generator=self._generator)
            for idx in order.chunk(self.config.num_minibatches):
                loss, t = self._loss({k: v[idx] for k, v in flat.items()})
                norm = self._apply(loss)
                out = {"loss": loss.detach().float(), "grad_norm": norm.detach(), **{k: v.detach() for k, v in t.items()}}
        out["learning_rate"] = self.optimizer.param_groups[0]["lr"]
        out["explained_variance"] = explained_variance(rollout["value"].flatten(), rollout["target"].flatten())
        return out

    def evaluate_loss(self, rollout: dict[str, Tensor]) -> Tensor:
        return self._loss({k: v.flatten(0, 1) for k, v in rollout.items()})[0].detach()


class CraftaxRNNTrainStep(_RolloutStep):
    """PPO on the GRU actor-critic (``priml/baselines/craftax/rnn_train_step.py``)."""

    class Config(Makes["CraftaxRNNTrainStep"], _RolloutStep.Config, kw_only=False):
        model: Any = field(default_factory=ActorCriticRNN.Config)
        rollout_steps: int = 64
        clip_epsilon: float = 0.2
        entropy_coefficient: float = 0.01
        value_coefficient: float = 0.5

    def __init__(self, config: Config) -> None:
        super().__init__(config)
        self._hidden = self.model.initial_state(self._observation.shape[0], self.device)

    @staticmethod
    def _parts(state: Any) -> tuple[Tensor, ...]:
        return tuple(state) if isinstance(state, tuple) else (state,)

    def _pack(self, parts: tuple[Tensor, ...]) -> Any:
        return parts if isinstance(self._hidden, tuple) else parts[0]

    def _keep_dtype(self, state: Any) -> Any:
        return self._pack(tuple(x.float() if x.is_floating_point() else x for x in self._parts(state)))

    @torch.no_grad()
    def collect(self) -> dict[str, Tensor]:
        h0 = {f"h0_{i}": x.clone()[None] for i, x in enumerate(self._parts(self._hidden))}
        obs, pdone, act, logp, val, rew, done = [], [], [], [], [], [], []
        for _ in range(self.config.rollout_steps):
            with self._autocast():
                self._hidden, logits, value = self.model.step(self._hidden, self._observation, self._done)
            self._hidden = self._keep_dtype(self._hidden)
            lp = logits.float().log_softmax(-1)
            a = torch.multinomial(lp.exp(), 1, generator=self._generator)[:, 0]
            obs.append(self._observation)
            pdone.append(self._done)
            act.append(a)
            logp.append(lp.gather(-1, a[:, None])[:, 0])
            val.append(value.float())
            t = self.env.step(a)
            self._observation, self._done = t.observation, t.done
            rew.append(t.reward)
            done.append(t.done)
            self._record(t.reward, t.done)
        with self._autocast():
            _, _, last = self.model.step(self._hidden, self._observation, self._done)
        value = torch.stack(val)
        adv, target = generalized_advantage(rewards=torch.stack(rew), values=value, dones=torch.stack(done),
                                            last_value=last.float(), discount=self.config.discount,
                                            trace_decay=self.config.trace_decay)  # fmt: skip
        return {"observation": torch.stack(obs), "previous_done": torch.stack(pdone), "action": torch.stack(act),
                "log_prob": torch.stack(logp), "value": value, "advantage": adv, "target": target, **h0}  # fmt: skip

    def _loss(self, mb: dict[str, Tensor]) -> tuple[Tensor, dict[str, Tensor]]:
        n = sum(1 for k in mb if k.startswith("h0_"))
        state = self._pack(tuple(mb[f"h0_{i}"][0] for i in range(n)))
        with self._autocast():
            _, logits, value = self.model.sequence(state, mb["observation"], mb["previous_done"])
        c = self.config
        t = ppo_terms(logits, mb["action"], mb["log_prob"], value, mb["value"], mb["advantage"], mb["target"],
                      c.clip_epsilon)  # fmt: skip
        return t["policy"] + c.value_coefficient * t["value"] - c.entropy_coefficient * t["entropy"], t

    def optimize(self, rollout: dict[str, Tensor]) -> dict[str, Any]:
        n = rollout["action"].shape[1]
        out: dict[str, Any] = {}
        for _ in range(self.config.num_epochs):
            order = torch.randperm(n, device=self.device, generator=self._generator)
            for idx in order.chunk(self.config.num_minibatches):
                loss, t = self._loss({k: v[:, idx] for k, v in rollout.items()})
                norm = self._apply(loss)
                out = {"loss": loss.detach().float(), "grad_norm": norm.detach(), **{k: v.detach() for k, v in t.items()}}
        out["learning_rate"] = self.optimizer.param_groups[0]["lr"]
        out["explained_variance"] = explained_variance(rollout["value"].flatten(), rollout["target"].flatten())
        return out

    def evaluate_loss(self, rollout: dict[str, Tensor]) -> Tensor:
        return self._loss(rollout)[0].detach()

    def state_dict(self) -> dict[str, Any]:
        return super().state_dict() | {"hidden": self._hidden}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        super().load_state_dict(s)
        self._hidden = s["hidden"]


class CraftaxGTrXLTrainStep(CraftaxRNNTrainStep):
    """PPO on the gated Transformer-XL policy (``priml/baselines/craftax/gtrxl_train_step.py``): the
    same recurrent machinery, with a memory of the last 128 inputs per layer as the carried state."""

    class Config(Makes["CraftaxGTrXLTrainStep"], CraftaxRNNTrainStep.Config, kw_only=False):
        model: Any = field(default_factory=ActorCriticGTrXL.Config)
        rollout_steps: int = 128


class CraftaxPQNTrainStep(_RolloutStep):
    """PQN on the recurrent Q-network (``priml/baselines/craftax/pqn_train_step.py``)."""

    class Config(Makes["CraftaxPQNTrainStep"], _RolloutStep.Config, kw_only=False):
        model: Any = field(default_factory=RecurrentQNetwork.Config)
        rollout_steps: int = 128
        num_minibatches: int = 4
        total_train_steps: int = 7629
        trace_decay: float = 0.5
        epsilon_start: float = 1.0
        epsilon_finish: float = 0.005
        epsilon_decay_fraction: float = 0.1
        max_grad_norm: float = 0.5

        def _optimizer(self) -> Any:
            return PartialConfig(torch.optim.RAdam, lr=self.learning_rate)

    def __init__(self, config: Config) -> None:
        super().__init__(config)
        self._state = self.model.initial_state(self._observation.shape[0], self.device)
        self._prev_action = torch.zeros(self._observation.shape[0], dtype=torch.long, device=self.device)

    @torch.no_grad()
    def collect(self) -> dict[str, Tensor]:
        c = self.config
        eps = epsilon_at(self.global_step, total_updates=c.total_train_steps, start=c.epsilon_start,
                         finish=c.epsilon_finish, decay_fraction=c.epsilon_decay_fraction)  # fmt: skip
        s0 = (self._state[0].clone(), self._state[1].clone())
        obs, pact, pdone, act, rew, done, qs = [], [], [], [], [], [], []
        self.model.eval()  # batch statistics are not updated by acting
        for _ in range(c.rollout_steps):
            with self._autocast():
                self._state, q = self.model.step(self._state, self._observation, self._prev_action, self._done)
            self._state = (self._state[0].float(), self._state[1].float())
            greedy = q.float().argmax(-1)
            explore = torch.rand(greedy.shape, device=self.device, generator=self._generator) < eps
            rand = torch.randint(0, q.shape[-1], greedy.shape, device=self.device, generator=self._generator)
            a = torch.where(explore, rand, greedy)
            obs.append(self._observation)
            pact.append(self._prev_action)
            pdone.append(self._done)
            act.append(a)
            qs.append(q.float())
            t = self.env.step(a)
            self._observation, self._done, self._prev_action = t.observation, t.done, a
            rew.append(t.reward)
            done.append(t.done)
            self._record(t.reward, t.done)
        with self._autocast():
            _, last_q = self.model.step(self._state, self._observation, self._prev_action, self._done)
        self.model.train()
        q_all = torch.stack(qs + [last_q.float()])
        target = q_lambda_targets(rewards=torch.stack(rew), q_values=q_all, dones=torch.stack(done),
                                  discount=c.discount, trace_decay=c.trace_decay)  # fmt: skip
        return {"observation": torch.stack(obs), "previous_action": torch.stack(pact),
                "previous_done": torch.stack(pdone), "action": torch.stack(act), "target": target,
                "s0h": s0[0][None], "s0c": s0[1][None], "epsilon": torch.tensor([eps], device=self.device)}  # fmt: skip

    def _loss(self, mb: dict[str, Tensor]) -> Tensor:
        with self._autocast():
            _, q = self.model.sequence((mb["s0h"][0], mb["s0c"][0]), mb["observation"], mb["previous_action"],
                                       mb["previous_done"])  # fmt: skip
        chosen = q.float().gather(-1, mb["action"][..., None])[..., 0]
        return 0.5 * F.mse_loss(chosen, mb["target"])

    def optimize(self, rollout: dict[str, Tensor]) -> dict[str, Any]:
        n = rollout["action"].shape[1]
        eps = rollout.pop("epsilon")
        out: dict[str, Any] = {}
        for _ in range(self.config.num_epochs):
            order = torch.randperm(n, device=self.device, generator=self._generator)
            for idx in order.chunk(self.config.num_minibatches):
                loss = self._loss({k: v[:, idx] for k, v in rollout.items()})
                norm = self._apply(loss)
                out = {"loss": loss.detach(), "grad_norm": norm.detach()}
        out["learning_rate"] = self.optimizer.param_groups[0]["lr"]
        out["epsilon"] = eps[0]
        return out

    def evaluate_loss(self, rollout: dict[str, Tensor]) -> Tensor:
        rollout.pop("epsilon", None)
        return self._loss(rollout).detach()

    def state_dict(self) -> dict[str, Any]:
        return super().state_dict() | {"q_state": self._state, "previous_action": self._prev_action}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        super().load_state_dict(s)
        self._state, self._prev_action = s["q_state"], s["previous_action"]
