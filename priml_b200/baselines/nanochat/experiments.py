"""NanoChat experiment ladder (``priml/baselines/nanochat/experiments.py:55-403``).

``NanoChatLoop`` stops on, reports and anneals against ONE clock, the train
step's budget clock (warmup excluded, batch fetching charged), and wires the
dataset's batch size, vocabulary and row length from the step's model.

* ``exp000`` -- the published five-minute recipe: d512, 8 layers, SSSL windows,
  value embeddings on alternating layers, bf16 tables and rotary factors,
  eps = fp32 epsilon RMS norms, 300 s budget, one bits-per-byte eval at the end.
  The reference pins FlashAttention-3 (sm_90 only); on B200 the attention is
  this package's tcgen05 flash-attention kernel with the same windows.
* ``exp001`` -- the same recipe through ATen SDPA (the portable kernel).
* ``exp002`` -- exp001 without value embeddings.
* ``exp003`` -- exp002 with every layer attending over the full context.
* ``exp_smoke`` -- exp001 at minimum size, for checking an installation.

Run: ``python -m priml_b200 priml_b200.baselines.nanochat.experiments.exp000``.
"""

from __future__ import annotations

from dataclasses import field
from typing import Any

import torch

from priml_b200.baselines.nanochat.data import NanoChatData
from priml_b200.baselines.nanochat.train_step import NanoChatTrainStep
from priml_b200.config import Makes, PartialConfig
from priml_b200.metrics import BitsPerByte
from priml_b200.models.embedding import NarrowEmbedding
from priml_b200.models.norm import RMSNorm
from priml_b200.models.value_gated_attention import ValueGatedAttention
from priml_b200.parallel.runtime import SingleProcess
from priml_b200.parallel.strategies import NoParallel
from priml_b200.train.train_loop import TrainLoop

__all__ = ["NanoChatLoop", "exp000", "exp001", "exp002", "exp003", "exp_smoke"]


class NanoChatLoop(TrainLoop):
    """A loop whose time limit is the nanochat step's budget clock."""

    class Config(Makes["NanoChatLoop"], TrainLoop.Config):
        step: Any = field(default_factory=NanoChatTrainStep.Config)
        dataset: Any = field(default_factory=NanoChatData.Config)

        def finalize(self):  # noqa: ANN201
            self.dataset.batch_size = self.step.rows_per_pass
            self.dataset.vocab_size = self.step.model.vocab_size
            self.dataset.max_seq_len = self.step.model.max_seq_len
            return super().finalize()

    def _train_elapsed(self) -> float:
        return float(self.step.elapsed_sec)

    def _on_batch_ready(self, fetch_time: float) -> None:
        self.step.charge_budget(fetch_time)


def _template(cfg: NanoChatLoop.Config) -> Any:
    block = cfg.step.model.block
    return block[0] if isinstance(block, list) else block


def exp000() -> NanoChatLoop.Config:
    """The published recipe (see the module docstring)."""
    cfg = NanoChatLoop.Config()
    cfg.study_name = "nanochat"
    cfg.experiment_name = "exp000"
    block = _template(cfg)
    assert isinstance(block.attn, ValueGatedAttention.Config)
    # the reference's bare F.rms_norm leaves eps to torch: fp32 epsilon
    for norm in (block.norm1, block.norm2, block.attn.norm_qk):
        if isinstance(norm, RMSNorm.Config):
            norm.eps = torch.finfo(torch.float32).eps
    embedding = cfg.step.model.embedding
    assert isinstance(embedding, NarrowEmbedding.Config)
    embedding.dtype = torch.bfloat16
    cfg.step.model.rope.dtype = torch.bfloat16
    cfg.step.model.channels_in = 512
    cfg.step.model.num_layers = 8
    block.attn.window_pattern = "SSSL"
    cfg.step.model.value_embedding_stride = 2
    cfg.step.train_budget_sec = 300.0
    cfg.max_time = cfg.step.train_budget_sec
    cfg.max_time_kind = "train"
    cfg.metrics["val"] = BitsPerByte.Config()
    cfg.num_steps_eval = -1  # one eval, at the end
    cfg.num_steps_log = 1
    cfg.early_train_log_steps = 0
    cfg.eval_every_epoch = False
    cfg.seed = 42
    cfg.step.parallelism = NoParallel.Config()
    cfg.dataset.device = "cuda"
    cfg.runtime = SingleProcess.Config()
    return cfg


def exp001() -> NanoChatLoop.Config:
    """exp000 through ATen SDPA (the portable attention)."""
    from priml_b200.models.value_gated_attention import sdpa_attention

    cfg = exp000()
    cfg.experiment_name = "exp001"
    _template(cfg).attn.kernel = PartialConfig(sdpa_attention)
    return cfg


def exp002() -> NanoChatLoop.Config:
    """exp001 without the value embeddings."""
    cfg = exp001()
    cfg.experiment_name = "exp002"
    cfg.step.model.value_embedding_stride = 0
    return cfg


def exp003() -> NanoChatLoop.Config:
    """exp002 with every layer attending over the full context."""
    cfg = exp002()
    cfg.experiment_name = "exp003"
    _template(cfg).attn.window_pattern = "L"
    return cfg


def exp_smoke() -> NanoChatLoop.Config:
    """exp001 at minimum size: does the data load and the loop run."""
    cfg = exp001()
    cfg.experiment_name = "exp_smoke"
    cfg.dataset.device = "auto"
    cfg.step.model.vocab_size = 16
    cfg.step.model.channels_in = 32
    cfg.step.model.num_layers = 2
    cfg.step.model.max_seq_len = 8
    _template(cfg).attn.channels_head = 16
    cfg.step.rows_per_pass = 2
    cfg.step.tokens_per_optimizer_step = 32
    cfg.step.budget_warmup_steps = 0
    cfg.step.train_budget_sec = 10.0
    cfg.max_time = cfg.step.train_budget_sec
    cfg.max_steps = 4
    cfg.num_steps_eval = 2
    cfg.dataset.eval_batch_size = 4
    cfg.dataset.eval_tokens = 2 * 4 * cfg.step.model.max_seq_len
    return cfg
