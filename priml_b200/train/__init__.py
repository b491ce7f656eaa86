"""Training orchestration (``priml/train/__init__.py``)."""

from priml_b200.parallel.strategies import (
    DataParallel,
    FullySharded,
    HybridSharded,
    NoParallel,
    RecursiveFullySharded,
    materialize_meta,
)
from priml_b200.parallel.tensor_parallel import TensorParallel, apply_tensor_parallel
from priml_b200.train.activation import (
    DefaultActivationStorage,
    Float8ActivationStorage,
    LayerActivationCheckpointing,
    QuantizedActivationStorage,
    QuantizedModuleActivationStorage,
    SelectiveActivationCheckpointing,
)
from priml_b200.train.checkpointing import AsyncLocalStateDictStorer, Checkpointer, SyncLocalStateDictStorer
from priml_b200.train.ema import EMA, NoEMA, karras_decay
from priml_b200.train.profiling import PhaseTimer, TorchProfiling
from priml_b200.train.tracker import AsyncTracker, FileTracker, NoTracker, TensorBoardTracker, TrackerList, WandbTracker
from priml_b200.train.train_loop import EvalTimeLimitError, TrainLoop
from priml_b200.train.progress import write_progress
from priml_b200.train.quantization import Float8ModelQuantization, NoModelQuantization
from priml_b200.train.results import format_summary, read_metrics, summarize
from priml_b200.train.train_step import TrainStep, TrainStepOutput
from priml_b200.train.train_step_gan import GANTrainStep

__all__ = [
    "Float8ModelQuantization",
    "NoModelQuantization",
    "GANTrainStep",
    "format_summary",
    "read_metrics",
    "summarize",
    "write_progress",
    "EMA",
    "AsyncLocalStateDictStorer",
    "AsyncTracker",
    "Checkpointer",
    "DataParallel",
    "DefaultActivationStorage",
    "EvalTimeLimitError",
    "FileTracker",
    "Float8ActivationStorage",
    "FullySharded",
    "HybridSharded",
    "LayerActivationCheckpointing",
    "QuantizedActivationStorage",
    "QuantizedModuleActivationStorage",
    "NoEMA",
    "NoParallel",
    "NoTracker",
    "PhaseTimer",
    "RecursiveFullySharded",
    "SelectiveActivationCheckpointing",
    "SyncLocalStateDictStorer",
    "TensorBoardTracker",
    "TensorParallel",
    "TorchProfiling",
    "TrackerList",
    "TrainLoop",
    "TrainStep",
    "TrainStepOutput",
    "WandbTracker",
    "apply_tensor_parallel",
    "karras_decay",
    "materialize_meta",
]
