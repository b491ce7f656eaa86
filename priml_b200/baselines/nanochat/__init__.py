"""NanoChat: Karpathy's five-minute language-model recipe (``priml/baselines/nanochat``)."""

from priml_b200.baselines.nanochat.model import NanoChatLM
from priml_b200.baselines.nanochat.train_step import NanoChatTrainStep, nanochat_loss, nanochat_optimizer

__all__ = ["NanoChatLM", "NanoChatTrainStep", "nanochat_loss", "nanochat_optimizer"]
