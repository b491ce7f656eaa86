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

__all__ = ["ActorCritic", "ActorCriticGTrXL", "ActorCriticRNN", "RecurrentQNetwork", "epsilon_at"]

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


class _Gate(nn.Module):
    """GRU-style gating of a residual branch (Parisotto et al. 2019): ``(1 - z) x + z h``."""

    def __init__(self, d: int, bias: float) -> None:
        super().__init__()
        self.wy = nn.Linear(d, 3 * d, bias=False)
        self.ux = nn.Linear(d, 2 * d, bias=False)
        self.ug = nn.Linear(d, d, bias=False)
        self.bias = bias

    def forward(self, x: Tensor, y: Tensor) -> Tensor:
        wr, wz, wg = self.wy(y).chunk(3, -1)
        ur, uz = self.ux(x).chunk(2, -1)
        r = torch.sigmoid(wr + ur)
        z = torch.sigmoid(wz + uz - self.bias)
        h = torch.tanh(wg + self.ug(r * x))
        return (1 - z) * x + z * h


class _GTrXLLayer(nn.Module):
    def __init__(self, d: int, heads: int, gating_bias: float) -> None:
        super().__init__()
        self.heads = heads
        self.norm1, self.norm2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.q = nn.Linear(d, d, bias=False)
        self.kv = nn.Linear(d, 2 * d, bias=False)
        self.o = nn.Linear(d, d, bias=False)
        self.mlp = nn.Sequential(nn.Linear(d, d), nn.ReLU(), nn.Linear(d, d))
        self.gate1, self.gate2 = _Gate(d, gating_bias), _Gate(d, gating_bias)

    def forward(self, x: Tensor, memory: Tensor, valid: Tensor, positions: Tensor) -> Tensor:
        """``x`` [E, D] (this step), ``memory`` [E, M, D] (earlier inputs), ``valid`` [E, M + 1] key mask."""
        e, m, d = memory.shape
        h = self.heads
        keys = self.norm1(torch.cat([memory, x[:, None]], 1)) + positions
        q = self.q(keys[:, -1]).view(e, h, 1, d // h)
        k, v = self.kv(keys).view(e, m + 1, 2, h, d // h).unbind(2)
        att = torch.nn.functional.scaled_dot_product_attention(q, k.transpose(1, 2), v.transpose(1, 2),
                                                               attn_mask=valid[:, None, None, :])  # fmt: skip
        x = self.gate1(x, torch.relu(self.o(att.reshape(e, d))))
        return self.gate2(x, torch.relu(self.mlp(self.norm2(x))))


def _sinusoid(length: int, d: int, device: torch.device) -> Tensor:
    pos = torch.arange(length, device=device, dtype=torch.float32)[:, None]
    freq = torch.exp(torch.arange(0, d, 2, device=device, dtype=torch.float32) * (-math.log(10000.0) / d))
    out = torch.zeros(length, d, device=device)
    out[:, 0::2], out[:, 1::2] = torch.sin(pos * freq), torch.cos(pos * freq)
    return out


class ActorCriticGTrXL(nn.Module):
    """Gated Transformer-XL policy: each step attends over the last ``memory_length`` inputs of
    every layer (reset at episode boundaries), with GRU-gated residuals and sinusoidal positions
    (oldest memory slot first). Recurrent state: (memory [E, L, M, D], filled length [E])."""

    class Config(Fig["ActorCriticGTrXL"]):
        observation_size: int = _OBS
        num_actions: int = _ACTIONS
        embed_dim: int = 256
        num_heads: int = 8
        num_layers: int = 2
        hidden_size: int = 256
        memory_length: int = 128
        gating_bias: float = 2.0

    def __init__(self, config: Config) -> None:
        super().__init__()
        c = config
        if c.embed_dim % c.num_heads or min(c.memory_length, c.num_layers) <= 0:
            raise ValueError("embed_dim must divide into heads; memory_length and num_layers must be positive")
        self.c = c
        self.embed = nn.Sequential(_dense(c.observation_size, c.embed_dim, math.sqrt(2.0)), nn.ReLU())
        self.layers = nn.ModuleList(_GTrXLLayer(c.embed_dim, c.num_heads, c.gating_bias) for _ in range(c.num_layers))
        self.actor = _tower(c.embed_dim, c.hidden_size, 2, c.num_actions, 0.01, nn.ReLU)
        self.critic = _tower(c.embed_dim, c.hidden_size, 2, 1, 1.0, nn.ReLU)

    def initial_state(self, n: int, device: torch.device | str = "cpu") -> tuple[Tensor, Tensor]:
        c = self.c
        return (torch.zeros(n, c.num_layers, c.memory_length, c.embed_dim, device=device),
                torch.zeros(n, dtype=torch.long, device=device))  # fmt: skip

    def step(self, state: tuple[Tensor, Tensor], observation: Tensor,
             previous_done: Tensor) -> tuple[tuple[Tensor, Tensor], Tensor, Tensor]:  # fmt: skip
        memory, filled = state
        m = self.c.memory_length
        filled = torch.where(previous_done, torch.zeros_like(filled), filled)
        slot = torch.arange(m + 1, device=observation.device)
        valid = slot[None] >= (m - filled)[:, None]  # the newest `filled` memory slots and the current step
        positions = _sinusoid(m + 1, self.c.embed_dim, observation.device)
        x = self.embed(observation)
        inputs = []
        for i, layer in enumerate(self.layers):
            inputs.append(x)
            x = layer(x, memory[:, i].to(x.dtype), valid, positions.to(x.dtype))
        new = torch.stack(inputs, 1).to(memory.dtype)[:, :, None]  # [E, L, 1, D]
        memory = torch.cat([memory[:, :, 1:], new], 2)
        return (memory, (filled + 1).clamp(max=m)), self.actor(x), self.critic(x).squeeze(-1)

    def sequence(self, state: tuple[Tensor, Tensor], observation: Tensor,
                 previous_done: Tensor) -> tuple[tuple[Tensor, Tensor], Tensor, Tensor]:  # fmt: skip
        logits, values = [], []
        for t in range(observation.shape[0]):
            state, lg, v = self.step(state, observation[t], previous_done[t])
            logits.append(lg)
            values.append(v)
        return state, torch.stack(logits), torch.stack(values)

    def forward(self, observation: Tensor) -> tuple[Tensor, Tensor]:
        n = observation.shape[0]
        done = torch.zeros(n, dtype=torch.bool, device=observation.device)
        _, logits, value = self.step(self.initial_state(n, observation.device), observation, done)
        return logits, value
