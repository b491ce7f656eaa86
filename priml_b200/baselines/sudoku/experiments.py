"""Sudoku experiment lattice (``priml/baselines/sudoku/experiments.py:1-223``).

Two axes vary independently, each a config VALUE on one model and one step:

==========  ===========  ===========
            transformer  MLP-mixer
==========  ===========  ===========
plain       ``exp000``   ``exp001``
recurrent   ``exp002``   ``exp003``
==========  ===========  ===========

``exp000``: hidden 512, 2 post-norm transformer blocks, factored row/column/box
positions, batch 384, 19,500 steps, Muon + AdamW, EMA 0.999, exact-grid and cell
accuracy on a 2,000-puzzle test prefix every 1,000 steps. The recurrent rungs add
a 6 x 9 deep recurrence, the prediction-feedback channel and an ACT pool of 384
slots (at most 32 steps). ``exp_smoke`` only checks that the data is prepared and
the loop runs.
"""

from __future__ import annotations

from dataclasses import field
from typing import Any, Final

from priml_b200.baselines.sudoku.act import ActPool
from priml_b200.baselines.sudoku.data import SudokuData
from priml_b200.baselines.sudoku.embedding import FactoredPositions, GridEmbedding, PredictionFeedback
from priml_b200.baselines.sudoku.metric import GridAccuracy
from priml_b200.baselines.sudoku.model import DeepRecurrence
from priml_b200.baselines.sudoku.train_step import SudokuTrainStep
from priml_b200.config import Makes
from priml_b200.models.norm import RMSNorm
from priml_b200.models.swiglu import SwiGLU
from priml_b200.models.vision import MLPMixerBlock
from priml_b200.parallel.runtime import SingleProcess
from priml_b200.train.train_loop import TrainLoop

__all__ = ["GRID_LEN", "SudokuTrainLoop", "exp000", "exp001", "exp002", "exp003", "exp_smoke", "mixer_block"]

GRID_LEN: Final = 81


class SudokuTrainLoop(Makes["TrainLoop"], TrainLoop.Config):
    step: Any = field(default_factory=SudokuTrainStep.Config)
    dataset: Any = field(default_factory=SudokuData.Config)


def mixer_block(seq_len: int) -> MLPMixerBlock.Config:
    """Post-norm mixer block with RMS-normalized SwiGLU token and channel mixers."""
    return MLPMixerBlock.Config(seq_len=seq_len, prenorm=False, token_mixer=SwiGLU.Config(norm=RMSNorm.Config()),
                                channel_mixer=SwiGLU.Config(norm=RMSNorm.Config()))  # fmt: skip


def exp000() -> SudokuTrainLoop:
    cfg = SudokuTrainLoop()
    cfg.study_name = "sudoku"
    cfg.experiment_name = "exp000"
    emb = GridEmbedding.Config()
    emb.channels = [FactoredPositions.Config()]
    cfg.step.model.embedding = emb
    cfg.step.model.hidden_size = 512
    cfg.step.model.num_layers = 2
    cfg.dataset.batch_size = 384
    cfg.dataset.seed = 0
    cfg.dataset.num_eval_puzzles = 2000
    cfg.metrics["accuracy"] = GridAccuracy.Config()
    cfg.max_steps = cfg.step.total_train_steps = 19500
    cfg.num_steps_eval = 1000
    cfg.runtime = SingleProcess.Config()
    return cfg


def exp001() -> SudokuTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp001"
    cfg.step.model.block = mixer_block(GRID_LEN)
    return cfg


def exp002() -> SudokuTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp002"
    cfg.step.model.recurrence = DeepRecurrence.Config()
    cfg.step.model.embedding.channels = [FactoredPositions.Config(), PredictionFeedback.Config()]
    cfg.step.act = ActPool.Config(batch_size=cfg.dataset.batch_size)
    return cfg


def exp003() -> SudokuTrainLoop:
    cfg = exp002()
    cfg.experiment_name = "exp003"
    cfg.step.model.block = mixer_block(GRID_LEN)
    return cfg


def exp_smoke() -> SudokuTrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp_smoke"
    cfg.step.model.hidden_size = 32
    cfg.step.model.num_layers = 1
    cfg.dataset.batch_size = 8
    cfg.dataset.num_train_puzzles = 4
    cfg.dataset.num_eval_puzzles = 4
    cfg.max_steps = cfg.step.total_train_steps = 4
    cfg.num_steps_eval = 2
    return cfg
