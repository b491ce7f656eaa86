"""Craftax networks (``priml/baselines/craftax/model.py``, ``rnn.py``, ``pqn.py``).

* :class:`ActorCritic` -- separate policy and value towers (3 x 512 tanh layers,
  orthogonal init with gain sqrt(2), policy head gain 0.01, value head gain 1):
  the PPO baseline's network.
* :class:`ActorCriticRNN` -- a ReLU embedding, a GRU cell whose state is zeroed
  where the previous step ended an episode, and two 2-layer ReLU heads.
* :class:`RecurrentQNetwork` -- PQN's network: batch-renormalized input, a
  LayerNorm'd ReLU encoder, an LSTM cell fed the encoding and the previous
  action (one-hot), and a linear Q head.

The dense layers are :class:`priml_b200.models.linear.Linear` (the tcgen05 GEMM
on CUDA under bf16 autocast); the GRU / LSTM cells are torch's.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor, nn

from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game.observation import observation_size
from priml_b200.config import Fig
from priml_b200.models.linear import Linear
from priml_b200.models.norm import BatchRenorm

__all__ = ["ActorCritic", "ActorCriticRNN", "RecurrentQNetwork", "epsilon_at"]

_OBS = observation_size()
_ACTIONS = len(C.Action)


def _dense(n_in: int, n_out: int, gain: float) -> nn.Linear:
    layer = Linear.Config(n_in, n_out, bias=True).make()
    with torch.no_grad():
        nn.init.orthogonal_(layer.weight, gain=gain)
        nn.init.zeros_(layer.bias)
    return layer


def _tower(n_in: int, hidden: int, layers: int, n_out: int, out_gain: float, act: type[nn.Module]) -> nn.Sequential:
    mods: list[nn.Module] = []
    width = n_in
    for _ in range(layers):
        mods += [_dense(width, hidden, math.sqrt(2.0)), act()]
        width = hidden
    mods.append(_dense(width, n_out, out_gain))
    return nn.Sequential(*mods)


class ActorCritic(nn.Module):
    class Config(Fig["ActorCritic"]):
        observation_size: int = _OBS
        num_actions: int = _ACTIONS
        hidden_size: int = 512
        num_layers: int = 3

    def __init__(self, config: Config) -> None:
        super().__init__()
        if min(config.observation_size, config.num_actions, config.hidden_size, config.num_layers) <= 0:
            raise ValueError("ActorCritic dimensions must be positive")
        c = config
        self.policy = _tower(c.observation_size, c.hidden_size, c.num_layers, c.num_actions, 0.01, nn.Tanh)
        self.value = _tower(c.observation_size, c.hidden_size, c.num_layers, 1, 1.0, nn.Tanh)

    def forward(self, observation: Tensor) -> tuple[Tensor, Tensor]:
        return self.policy(observation), self.value(observation).squeeze(-1)


class ActorCriticRNN(nn.Module):
    class Config(Fig["ActorCriticRNN"]):
        observation_size: int = _OBS
        num_actions: int = _ACTIONS
        hidden_size: int = 512

    def __init__(self, config: Config) -> None:
        super().__init__()
        h = config.hidden_size
        if min(config.observation_size, config.num_actions, h) <= 0:
            raise ValueError("ActorCriticRNN dimensions must be positive")
        self.hidden_size = h
        self.embed = nn.Sequential(_dense(config.observation_size, h, math.sqrt(2.0)), nn.ReLU())
        self.cell = nn.GRUCell(h, h)
        self.actor = _tower(h, h, 2, config.num_actions, 0.01, nn.ReLU)
        self.critic = _tower(h, h, 2, 1, 1.0, nn.ReLU)

    def initial_state(self, n: int, device: torch.device | str = "cpu") -> Tensor:
        return torch.zeros(n, self.hidden_size, device=device)

    def step(self, state: Tensor, observation: Tensor, previous_done: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        state = self.cell(self.embed(observation), state * (~previous_done)[:, None].to(state.dtype))
        return state, self.actor(state), self.critic(state).squeeze(-1)

    def sequence(self, state: Tensor, observation: Tensor, previous_done: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        """``[T, E, ...]`` inputs; the embedding of all steps is one batched GEMM, the cell runs in order."""
        t, e = observation.shape[:2]
        embedded = self.embed(observation.flatten(0, 1)).view(t, e, -1)
        states = []
        for i in range(t):
            state = self.cell(embedded[i], state * (~previous_done[i])[:, None].to(state.dtype))
            states.append(state)
        hs = torch.stack(states)
        return state, self.actor(hs), self.critic(hs).squeeze(-1)

    def forward(self, observation: Tensor) -> tuple[Tensor, Tensor]:
        n = observation.shape[0]
        done = torch.zeros(n, dtype=torch.bool, device=observation.device)
        _, logits, value = self.step(self.initial_state(n, observation.device), observation, done)
        return logits, value


class RecurrentQNetwork(nn.Module):
    class Config(Fig["RecurrentQNetwork"]):
        observation_size: int = _OBS
        num_actions: int = _ACTIONS
        hidden_size: int = 512

    def __init__(self, config: Config) -> None:
        super().__init__()
        h = config.hidden_size
        if min(config.observation_size, config.num_actions, h) <= 0:
            raise ValueError("RecurrentQNetwork dimensions must be positive")
        self.hidden_size, self.num_actions = h, config.num_actions
        self.normalize = BatchRenorm.Config(channels_in=config.observation_size).make()
        self.encoder = Linear.Config(config.observation_size, h, bias=True).make()
        self.encoder_norm = nn.LayerNorm(h)
        self.cell = nn.LSTMCell(h + config.num_actions, h)
        self.head = Linear.Config(h, config.num_actions, bias=True).make()

    def initial_state(self, n: int, device: torch.device | str = "cpu") -> tuple[Tensor, Tensor]:
        z = torch.zeros(n, self.hidden_size, device=device)
        return z, z.clone()

    def _encode(self, observation: Tensor, previous_action: Tensor) -> Tensor:
        x = self.encoder_norm(self.encoder(self.normalize(observation))).relu()
        return torch.cat([x, nn.functional.one_hot(previous_action.long(), self.num_actions).to(x.dtype)], -1)

    def step(self, state: tuple[Tensor, Tensor], observation: Tensor, previous_action: Tensor,
             previous_done: Tensor) -> tuple[tuple[Tensor, Tensor], Tensor]:  # fmt: skip
        keep = (~previous_done)[:, None].to(state[0].dtype)
        h, c = self.cell(self._encode(observation, previous_action), (state[0] * keep, state[1] * keep))
        return (h, c), self.head(h)

    def sequence(self, state: tuple[Tensor, Tensor], observation: Tensor, previous_action: Tensor,
                 previous_done: Tensor) -> tuple[tuple[Tensor, Tensor], Tensor]:  # fmt: skip
        t, e = observation.shape[:2]
        enc = self._encode(observation.flatten(0, 1), previous_action.flatten(0, 1)).view(t, e, -1)
        hs = []
        for i in range(t):
            keep = (~previous_done[i])[:, None].to(state[0].dtype)
            state = self.cell(enc[i], (state[0] * keep, state[1] * keep))
            hs.append(state[0])
        return state, self.head(torch.stack(hs))

    def forward(self, observation: Tensor) -> Tensor:
        n = observation.shape[0]
        z = torch.zeros(n, dtype=torch.long, device=observation.device)
        return self.step(self.initial_state(n, observation.device), observation, z, z.bool())[1]


def epsilon_at(update: int, *, total_updates: int, start: float = 1.0, finish: float = 0.005,
               decay_fraction: float = 0.1) -> float:  # fmt: skip
    """Exploration rate: linear from ``start`` to ``finish`` over the first ``decay_fraction`` of the run."""
    if total_updates <= 0 or not 0.0 < decay_fraction <= 1.0:
        raise ValueError("total_updates must be positive and decay_fraction in (0, 1]")
    progress = min(1.0, update / max(1.0, decay_fraction * total_updates))
    return start + (finish - start) * progress
