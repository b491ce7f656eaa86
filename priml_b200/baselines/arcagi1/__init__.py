"""ARC-AGI-1 abstract reasoning (``priml/baselines/arcagi1``).

Each task demonstrates a rule with a few input/output grid pairs; the model
must apply it to a held-out input, scored whole-grid by pass@K. The solver,
recurrence, ACT pool and train step are the sudoku baseline's; this package
holds ARC's data, metric and experiment ladder.
"""

from priml_b200.baselines.arcagi1.data import ArcData
from priml_b200.baselines.arcagi1.metric import PassK

__all__ = ["ArcData", "PassK"]
