"""Craftax experiment chain (``priml/baselines/craftax/experiments.py``).

==========  ========  =========================================================
experiment  parent    change
==========  ========  =========================================================
``exp000``  --        PPO, 1M interactions: 256 workers x 16 steps, 244 updates
``exp001``  exp000    the published 1B recipe: 1024 workers x 64 steps, lr 2e-4
``exp002``  exp001    a reset-aware GRU policy (recurrent PPO)
``exp003``  exp001    no policy at all: PQN with an LSTM Q-network
``exp011``  exp001    the 1B geometry at 100M interactions (a screening budget)
``exp013``  exp001    a policy with memory, expensively: gated Transformer-XL
==========  ========  =========================================================

``exp_smoke`` cuts exp000 to a few updates. Evaluation plays the policy in fresh worlds (:class:`CraftaxScore`).
"""

from __future__ import annotations

from dataclasses import field
from typing import Any

from priml_b200.baselines.craftax.data import CraftaxRollouts
from priml_b200.baselines.craftax.metric import CraftaxScore
from priml_b200.baselines.craftax.train_step import (
    CraftaxGTrXLTrainStep,
    CraftaxPQNTrainStep,
    CraftaxRNNTrainStep,
    CraftaxTrainStep,
)
from priml_b200.config import Makes
from priml_b200.parallel.runtime import SingleProcess
from priml_b200.train.train_loop import TrainLoop

__all__ = ["CraftaxTrainLoop", "exp000", "exp001", "exp002", "exp003", "exp011", "exp013", "exp_smoke"]


class CraftaxTrainLoop(Makes["TrainLoop"], TrainLoop.Config):
    step: Any = field(default_factory=CraftaxTrainStep.Config)
    dataset: Any = field(default_factory=CraftaxRollouts.Config)


def _updates(interactions: int, envs: int, steps: int) -> int:
    return max(1, interactions // (envs * steps))


def exp000() -> CraftaxTrainLoop:
    cfg = CraftaxTrainLoop()
    cfg.study_name = "craftax"
    cfg.experiment_name = "exp000"
    cfg.step.env.num_envs = 256
    cfg.step.rollout_steps = 16
    cfg.max_steps = cfg.step.total_train_steps = _updates(1_000_000, 256, 16)
    cfg.num_steps_eval = cfg.max_steps
    cfg.eval_every_epoch = False
    cfg.metrics["craftax"] = CraftaxScore.Config()
    cfg.runtime = SingleProcess.Config()
    return cfg


def exp001() -> CraftaxTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp001"
    cfg.step.env.num_envs = 1024
    cfg.step.rollout_steps = 64
    cfg.step.learning_rate = 2e-4
    cfg.max_steps = cfg.step.total_train_steps = _updates(1_000_000_000, 1024, 64)
    cfg.num_steps_eval = 1000
    return cfg


def exp002() -> CraftaxTrainLoop:
    cfg = exp001()
    cfg.experiment_name = "exp002"
    rnn = CraftaxRNNTrainStep.Config()
    rnn.env, rnn.rollout_steps, rnn.learning_rate = cfg.step.env, 64, 2e-4
    rnn.total_train_steps = cfg.step.total_train_steps
    cfg.step = rnn
    return cfg


def exp003() -> CraftaxTrainLoop:
    cfg = exp001()
    cfg.experiment_name = "exp003"
    pqn = CraftaxPQNTrainStep.Config()
    pqn.env = cfg.step.env
    pqn.env.num_envs = 1024
    pqn.total_train_steps = _updates(1_000_000_000, 1024, pqn.rollout_steps)
    cfg.step = pqn
    cfg.max_steps = pqn.total_train_steps
    return cfg


def exp011() -> CraftaxTrainLoop:
    cfg = exp001()
    cfg.experiment_name = "exp011"
    cfg.max_steps = cfg.step.total_train_steps = _updates(100_000_000, 1024, 64)
    return cfg


def exp013() -> CraftaxTrainLoop:
    cfg = exp001()
    cfg.experiment_name = "exp013"
    gt = CraftaxGTrXLTrainStep.Config()
    gt.env, gt.learning_rate = cfg.step.env, 2e-4
    gt.total_train_steps = _updates(1_000_000_000, 1024, gt.rollout_steps)
    cfg.step = gt
    cfg.max_steps = gt.total_train_steps
    return cfg


def exp_smoke() -> CraftaxTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp_smoke"
    cfg.step.env.num_envs = 8
    cfg.step.rollout_steps = 4
    cfg.step.num_minibatches = 2
    cfg.max_steps = cfg.step.total_train_steps = 3
    cfg.num_steps_eval = 3
    cfg.metrics["craftax"] = CraftaxScore.Config(num_envs=4, steps=20)
    return cfg
