"""ARC-AGI-1 experiment ladder (``priml/baselines/arcagi1/experiments.py:1-268``).

The solver, recurrence, ACT pool and step are the sudoku baseline's, filled
with ARC's values: a 30 x 30 grid (900 tokens), 12 tokens, and a prefix of 16
per-puzzle tokens (a sparse table, one row per augmented view) plus one
register token that the halt head reads.

* ``exp000``: hidden 512, 2 post-norm transformer blocks, batch 256, 388,670
  steps with 2,000 warmup, EMA 0.999 after 2,000 steps, pass@K every 10,000
  steps, checkpoints every 4,000 steps (last 8 kept, every 40,000th forever).
* ``exp001``: the MLP-mixer block over the 917-token sequence.
* ``exp002``: a 3 x 4 deep recurrence, prediction feedback, an ACT pool of
  at most 16 steps with halt weight 0.5 (every color is a given).
* ``exp003``: ``exp002`` with the mixer block.
"""

from __future__ import annotations

from dataclasses import field
from typing import Any, Final

from priml_b200.baselines.arcagi1.data import ArcData, num_puzzle_identifiers
from priml_b200.baselines.arcagi1.metric import PassK
from priml_b200.baselines.sudoku.act import ActPool
from priml_b200.baselines.sudoku.embedding import GridEmbedding, PredictionFeedback
from priml_b200.baselines.sudoku.experiments import mixer_block
from priml_b200.baselines.sudoku.model import DeepRecurrence
from priml_b200.baselines.sudoku.prefix import PrefixStack, RegisterTokens, SparsePuzzleEmbedding
from priml_b200.baselines.sudoku.train_step import SudokuTrainStep
from priml_b200.config import Makes
from priml_b200.parallel.runtime import SingleProcess
from priml_b200.paths import resolve_working_dir
from priml_b200.train.checkpointing import Checkpointer
from priml_b200.train.train_loop import TrainLoop

__all__ = ["GRID_LEN", "VOCAB_SIZE", "ArcTrainLoop", "exp000", "exp001", "exp002", "exp003", "exp_smoke"]

GRID_LEN: Final = 900
VOCAB_SIZE: Final = 12


class ArcTrainLoop(Makes["TrainLoop"], TrainLoop.Config):
    step: Any = field(default_factory=SudokuTrainStep.Config)
    dataset: Any = field(default_factory=ArcData.Config)

    def finalize(self):  # noqa: ANN201
        # a per-puzzle table sized -1 takes its row count from the prepared data
        prefix = self.step.model.prefix
        for part in getattr(prefix, "parts", [prefix]):
            if isinstance(part, SparsePuzzleEmbedding.Config) and part.num_puzzles == -1:
                part.num_puzzles = num_puzzle_identifiers(resolve_working_dir(self.dataset.working_dir,
                                                                              self.dataset.base_dir))  # fmt: skip
        return super().finalize()


def exp000() -> ArcTrainLoop:
    cfg = ArcTrainLoop()
    cfg.study_name = "arcagi1"
    cfg.experiment_name = "exp000"
    cfg.seed = 0
    batch = 256
    m = cfg.step.model
    m.hidden_size = 512
    m.num_layers = 2
    m.vocab_size = VOCAB_SIZE
    m.embedding = GridEmbedding.Config(grid_shape=(GRID_LEN,))
    m.prefix = PrefixStack.Config(parts=[SparsePuzzleEmbedding.Config(num_puzzles=-1, num_tokens=16, batch_size=batch),
                                         RegisterTokens.Config(num_tokens=1)])  # fmt: skip
    cfg.step.total_train_steps = 388_670
    cfg.step.warmup_steps = 2000
    cfg.step.ema_decay = 0.999
    cfg.step.ema_warmup_steps = 2000
    cfg.dataset.batch_size = batch
    cfg.dataset.eval_batch_size = batch
    cfg.metrics["pass"] = PassK.Config()
    cfg.max_steps = cfg.step.total_train_steps
    cfg.num_steps_eval = 10_000
    cfg.num_steps_log = 100
    cfg.eval_warmup_batches = 1
    cfg.eval_every_epoch = False
    cfg.checkpointing = Checkpointer.Config(save_every=4000, keep_last_n=8, keep_every=40_000)
    cfg.runtime = SingleProcess.Config()
    return cfg


def exp001() -> ArcTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp001"
    cfg.step.model.block = mixer_block(cfg.step.model.total_seq_len)
    return cfg


def exp002() -> ArcTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp002"
    cfg.step.model.recurrence = DeepRecurrence.Config(slow_cycles=3, fast_cycles=4)
    cfg.step.model.embedding.channels = [PredictionFeedback.Config()]
    cfg.step.act = ActPool.Config(batch_size=cfg.dataset.batch_size, max_steps=16, halt_weight=0.5,
                                  given_high=VOCAB_SIZE - 1)  # fmt: skip
    return cfg


def exp003() -> ArcTrainLoop:
    cfg = exp002()
    cfg.experiment_name = "exp003"
    cfg.step.model.block = mixer_block(cfg.step.model.total_seq_len)
    return cfg


def exp_smoke() -> ArcTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp_smoke"
    cfg.step.model.hidden_size = 32
    cfg.step.model.num_layers = 1
    cfg.dataset.batch_size = 8
    cfg.dataset.eval_batch_size = 8
    cfg.dataset.num_tasks = 4
    cfg.max_steps = cfg.step.total_train_steps = 4
    cfg.num_steps_eval = 2
    cfg.checkpointing = None
    cfg.step.model.prefix.parts[0].batch_size = cfg.dataset.batch_size
    return cfg
