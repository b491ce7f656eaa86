"""Craftax: open-ended RL in a 2-D survival game (``priml/baselines/craftax``).

The game is a batched tensor program (``game/``); the learners are PPO,
recurrent (GRU) PPO, gated Transformer-XL PPO and PQN. This build covers the first two of the nine floors
(the overworld and the dungeon): terrain, tools and crafting, creatures and
projectiles, chests, bow, potions, attributes, survival meters, sleeping and
plants, with the full game's action space, achievement table (226-point
ceiling) and 8,268-float observation layout.
"""

from priml_b200.baselines.craftax.env import CraftaxEnv
from priml_b200.baselines.craftax.metric import CraftaxScore
from priml_b200.baselines.craftax.model import ActorCritic, ActorCriticGTrXL, ActorCriticRNN, RecurrentQNetwork
from priml_b200.baselines.craftax.train_step import (
    CraftaxGTrXLTrainStep,
    CraftaxPQNTrainStep,
    CraftaxRNNTrainStep,
    CraftaxTrainStep,
)

__all__ = ["ActorCritic", "ActorCriticGTrXL", "ActorCriticRNN", "CraftaxEnv", "CraftaxGTrXLTrainStep",
           "CraftaxPQNTrainStep", "CraftaxRNNTrainStep", "CraftaxScore", "CraftaxTrainStep", "RecurrentQNetwork"]
