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

from priml_b200.optimizers.misc import Newton
from priml_b200.parallel.strategies import RecursiveSharded
from priml_b200.train.custom_types import ModelQuantizationProtocol, ParallelStrategyProtocol

__all__ = [
    "AsyncLocalStateDictStorer",
    "AsyncTracker",
    "Checkpointer",
    "DataParallel",
    "DefaultActivationStorage",
    "EMA",
    "EvalTimeLimitError",
    "FileTracker",
    "Float8ActivationStorage",
    "Float8ModelQuantization",
    "FullySharded",
    "GANTrainStep",
    "HybridSharded",
    "LayerActivationCheckpointing",
    "ModelQuantizationProtocol",
    "Newton",
    "NoEMA",
    "NoModelQuantization",
    "NoParallel",
    "NoTracker",
    "ParallelStrategyProtocol",
    "PhaseTimer",
    "QuantizedActivationStorage",
    "QuantizedModuleActivationStorage",
    "RecursiveFullySharded",
    "RecursiveSharded",
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
    "format_summary",
    "karras_decay",
    "materialize_meta",
    "read_metrics",
    "summarize",
    "write_progress",
]
