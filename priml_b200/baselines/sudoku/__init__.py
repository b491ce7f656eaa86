"""Sudoku as whole-grid structured prediction (``priml/baselines/sudoku``).

The solver (:class:`SudokuNet`), its latent recurrence, the ACT pool and the
train step are generic over grid puzzles; the ARC-AGI baseline reuses them
with a different grid, vocabulary and prefix.
"""

from priml_b200.baselines.sudoku.act import ActPool
from priml_b200.baselines.sudoku.data import SudokuData, augment_sudoku
from priml_b200.baselines.sudoku.embedding import FactoredPositions, GridEmbedding, PredictionFeedback
from priml_b200.baselines.sudoku.metric import GridAccuracy
from priml_b200.baselines.sudoku.model import DeepRecurrence, ForwardOutput, SudokuNet
from priml_b200.baselines.sudoku.prefix import PrefixStack, RegisterTokens, SparsePuzzleEmbedding
from priml_b200.baselines.sudoku.train_step import SudokuTrainStep

__all__ = [
    "ActPool",
    "DeepRecurrence",
    "FactoredPositions",
    "ForwardOutput",
    "GridAccuracy",
    "GridEmbedding",
    "PredictionFeedback",
    "PrefixStack",
    "RegisterTokens",
    "SparsePuzzleEmbedding",
    "SudokuData",
    "SudokuNet",
    "SudokuTrainStep",
    "augment_sudoku",
]
