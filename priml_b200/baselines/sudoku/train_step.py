"""Train step shared by the grid-puzzle baselines (``priml/baselines/sudoku/train_step.py:1-490``).

One call is one optimizer step on one batch. Plain runs feed the batch through
the network once. With an :class:`ActPool`, the batch refills the halted slots
and every slot takes one recurrent step from its carried latents; the halt
head's BCE joins the token loss. The update is: backward -> optional clip ->
warmup + cosine learning-rate scale by ``global_step / total_train_steps`` ->
optimizer -> sparse puzzle-table update (when configured) -> EMA.

Losses: per-cell cross-entropy (fp32, optional label smoothing), averaged per
puzzle over counted cells, then over active slots.

Evaluation swaps in the EMA weights and, with a pool, rolls every puzzle out
for ``max_steps`` steps; its ``model`` output packs ``[halt, decoded grid]``
per row for :class:`GridAccuracy` and ``PassK``.

Differences from the reference, all deliberate:

* with ``act.feedback`` the pool's decoded grid also reaches the feedback
  channel during TRAINING (the reference computes it each step but feeds it
  only at evaluation, so a zero-initialized feedback table never trains);
* the pool seats each puzzle's identifier with the puzzle, so a slot that
  keeps an unsolved puzzle keeps reading ITS prefix row (the reference passes
  the incoming batch's identifiers to every slot);
* ``puzzle_optimizer`` (off by default, as in the reference) steps the sparse
  per-puzzle table with a sign-SGD sparse update.
"""

from __future__ import annotations

import contextlib
from collections.abc import Iterator
from dataclasses import field
from typing import Any

import torch
from torch import Tensor
from torch.nn import functional as F

from priml_b200.baselines.sudoku.act import ActPool
from priml_b200.baselines.sudoku.model import SudokuNet
from priml_b200.baselines.sudoku.prefix import SparsePuzzleEmbedding
from priml_b200.config import Makes
from priml_b200.optimizers import FusedAdamW, apply_lr_scale, lr_scale
from priml_b200.optimizers.composite import CompositeOptimizer, complement, excluding
from priml_b200.optimizers.muon import Muon
from priml_b200.train.ema import EMA, NoEMA
from priml_b200.train.train_step import TrainStep, TrainStepOutput

__all__ = ["SudokuTrainStep", "default_optimizer"]


def default_optimizer() -> CompositeOptimizer.Config:
    """Muon on the reasoning matrices, AdamW (decay 1.0) on tables, heads, norms and biases."""
    on_muon = excluding(Muon.eligible_tensor, "embed", "head")
    config = CompositeOptimizer.Config()
    config.optimizers = [
        FusedAdamW.Config(lr=1e-4, betas=(0.9, 0.95), weight_decay=1.0),
        Muon.Config(lr=0.02, momentum=0.6, nesterov=True, ns_steps=3),
    ]
    config.select = [complement(on_muon), on_muon]
    return config


def _prefix_kwargs(batch: dict[str, Any]) -> dict[str, Any]:
    ids = batch.get("puzzle_identifiers")
    return {} if ids is None else {"puzzle_identifiers": ids}


class SudokuTrainStep(TrainStep):
    class Config(Makes["SudokuTrainStep"], TrainStep.Config, kw_only=False):
        model: SudokuNet.Config = field(default_factory=SudokuNet.Config)
        optimizer: Any = field(default_factory=default_optimizer)
        dtype_autocast: torch.dtype | None = torch.bfloat16
        total_train_steps: int = 19500
        warmup_steps: int = 0
        lr_min_ratio: float = 0.0
        act: ActPool.Config | None = None
        label_smoothing: float = 0.0
        ignore_label_id: int = -100
        use_ema: bool = True
        ema_decay: float = 0.999
        ema_warmup_steps: int = 0
        """Steps during which the shadow copies the live weights."""
        puzzle_optimizer: Any = None
        """Optimizer config for the sparse per-puzzle tables (e.g. ``SignSGD.Config``); ``None`` leaves them fixed."""

        def finalize(self):  # noqa: ANN201
            if self.act is not None:
                self.act.grid_len = self.model.grid_len
                self.act.seq_len = self.model.total_seq_len
                self.act.hidden_size = self.model.hidden_size
            if self.use_ema:
                # a name-keyed param-dict shadow, seeded from the live weights when averaging starts
                self.ema = EMA.Config(decay=self.ema_decay, update_after_step=self.ema_warmup_steps,
                                      shadow_kind="param_dict", warmup_seed=True, track_buffers=False)  # fmt: skip
            else:
                self.ema = NoEMA.Config()
            return super().finalize()

    def __init__(self, config: Config) -> None:
        if config.total_train_steps <= 0:
            raise ValueError(f"total_train_steps must be positive; got {config.total_train_steps}.")
        super().__init__(config)
        self.config: SudokuTrainStep.Config = config
        self.act = config.act.make() if config.act is not None else None
        if self.act is not None:
            self.act.to(self.device)
        self.puzzle_tables = [m for m in self.model.modules() if isinstance(m, SparsePuzzleEmbedding)]
        self.puzzle_optimizer = None
        if config.puzzle_optimizer is not None and self.puzzle_tables:
            groups = [{"params": [t.weights, t.local_weights, t.local_ids], "sparse_embedding": True}
                      for t in self.puzzle_tables]  # fmt: skip
            self.puzzle_optimizer = config.puzzle_optimizer.make()(groups)
            for g in self.puzzle_optimizer.param_groups:
                g.setdefault("initial_lr", g["lr"])

    @property
    def net(self) -> SudokuNet:
        return self.model  # type: ignore[return-value]

    @property
    def global_step(self) -> int:
        return self.timer_step.global_count

    def progress_complete(self) -> float:
        return min(1.0, self.global_step / self.config.total_train_steps)

    @property
    def ema_shadow(self) -> dict[str, Tensor] | None:
        return self.ema.shadow_params if isinstance(self.ema, EMA) else None

    # ------------------------------------------------------------------ train
    def train_step(self, **batch: Any) -> TrainStepOutput:
        self.model.train()
        media, labels, active = self._ingest(batch)
        carry: tuple[Tensor, ...] = ()
        prefix = _prefix_kwargs(batch)
        if self.act is not None:
            carry = self.act.latents()
            if prefix:
                prefix = {"puzzle_identifiers": self.act.identifiers}
            if self.act.config.feedback:
                self.act.set_feedback(self.net, self.act.feedback)
        with self.timer_forward, self._autocast():
            out = self.net(media, *carry, **prefix)
            loss, metrics = self._loss(out.logits, labels=labels, halt=out.halt, active=active)
        loss.backward()
        with self.timer_step:
            norm = self._clip()
            if norm is not None:
                metrics["grad_norm"] = norm.detach()
            scale = lr_scale(self.global_step, self.config.total_train_steps, self.config.warmup_steps,
                             self.config.lr_min_ratio)  # fmt: skip
            apply_lr_scale([self.optimizer], scale)
            self.optimizer.step()
            self.optimizer.zero_grad(set_to_none=True)
            if self.puzzle_optimizer is not None:
                apply_lr_scale([self.puzzle_optimizer], scale)
                self.puzzle_optimizer.step()
            for t in self.puzzle_tables:
                t.local_weights.grad = None
            self.ema(self.model)
        metrics["lr"] = self.optimizer.param_groups[0]["lr"]
        if self.act is not None:
            self.act.advance(out.z_slow, z_fast=out.z_fast, logits=out.logits, halt=out.halt, media=media)
        self.last_loss = loss.detach()
        res = TrainStepOutput(loss=loss.detach().reshape(1), model=out.logits[:1, :1].detach(), metrics=metrics)
        res.update({k: v for k, v in metrics.items() if isinstance(v, Tensor)})
        res["num_samples"] = int(media.shape[0])
        res["stepped"] = True
        return res

    def train_loss(self, **batch: Any) -> TrainStepOutput:
        self.model.train()
        media, labels = batch["media"], batch["label"]
        with torch.no_grad(), self._autocast():
            out = self.net(media, **_prefix_kwargs(batch))
            active = torch.ones(media.shape[0], dtype=torch.bool, device=media.device)
            loss, metrics = self._loss(out.logits, labels=labels, halt=out.halt, active=active)
        return TrainStepOutput(loss=loss, model=out.logits, metrics=metrics)

    # ------------------------------------------------------------------ eval
    @contextlib.contextmanager
    def _eval_weights(self) -> Iterator[None]:
        if isinstance(self.ema, NoEMA) or self.global_step <= self.config.ema_warmup_steps:
            yield
            return
        with self.ema.apply_to(self.model):
            yield

    def _rollout(self, media: Tensor, prefix_kwargs: dict[str, Any]) -> tuple[Tensor, Tensor]:
        if self.act is None:
            out = self.net(media, **prefix_kwargs)
            return out.logits, out.halt
        return self.act.rollout(self.net, media=media, prefix_kwargs=prefix_kwargs)

    def eval_loss(self, **batch: Any) -> TrainStepOutput:
        media, labels = batch["media"], batch["label"]
        was_training = self.model.training
        self.model.eval()
        try:
            with self.timer_eval, self._eval_weights(), torch.inference_mode(), self._autocast():
                logits, halt = self._rollout(media, _prefix_kwargs(batch))
                active = torch.ones(media.shape[0], dtype=torch.bool, device=media.device)
                loss, metrics = self._loss(logits, labels=labels, halt=halt, active=active)
        finally:
            self.model.train(was_training)
        packed = torch.cat([halt.reshape(-1, 1).float(), logits.argmax(dim=-1).float()], dim=-1)
        return TrainStepOutput(loss=loss.detach().reshape(1), model=packed, metrics=metrics)

    def call_eval(self, *args: Any, **batch: Any) -> Tensor:
        media = args[0] if args else batch["media"]
        was_training = self.model.training
        self.model.eval()
        try:
            with self._eval_weights(), torch.inference_mode(), self._autocast():
                logits, _ = self._rollout(media, _prefix_kwargs(batch))
        finally:
            self.model.train(was_training)
        return logits

    def on_epoch_end(self) -> None:
        """Nothing to drop: every call is a complete optimizer step."""

    # ------------------------------------------------------------------ loss
    def _ingest(self, batch: dict[str, Any]) -> tuple[Tensor, Tensor, Tensor]:
        media, labels = batch["media"], batch["label"]
        if self.act is None:
            return media, labels, torch.ones(media.shape[0], dtype=torch.bool, device=media.device)
        valid = int(batch.get("valid_count", media.shape[0]))
        return self.act.refill(media, labels=labels, valid_count=valid, ignore_label_id=self.config.ignore_label_id,
                               identifiers=batch.get("puzzle_identifiers"))  # fmt: skip

    def _loss(self, logits: Tensor, *, labels: Tensor, halt: Tensor,
              active: Tensor) -> tuple[Tensor, dict[str, Any]]:  # fmt: skip
        c = self.config
        per_cell = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), labels.reshape(-1).long(),
                                   ignore_index=c.ignore_label_id, label_smoothing=c.label_smoothing,
                                   reduction="none").view(logits.shape[0], -1)  # fmt: skip
        counted = (labels != c.ignore_label_id).sum(-1).clamp(min=1)
        per_puzzle = per_cell.sum(-1) / counted
        lm = (per_puzzle * active).sum() / active.sum().clamp(min=1)
        metrics: dict[str, Any] = {"lm_loss": lm.detach()}
        if self.act is None:
            return lm, metrics
        halt_loss, more = self.act.halt_loss(logits, labels=labels, halt=halt, active=active,
                                             ignore_label_id=c.ignore_label_id)  # fmt: skip
        metrics.update(more)
        return lm + halt_loss, metrics

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict[str, Any]:
        s = super().state_dict()
        if self.act is not None:
            s["act"] = self.act.state_dict()
        if self.puzzle_optimizer is not None:
            s["puzzle_optimizer"] = self.puzzle_optimizer.state_dict()
        return s

    def load_state_dict(self, s: dict[str, Any]) -> None:
        super().load_state_dict(s)
        if self.act is not None and "act" in s:
            self.act.load_state_dict(s["act"])
        if self.puzzle_optimizer is not None and "puzzle_optimizer" in s:
            self.puzzle_optimizer.load_state_dict(s["puzzle_optimizer"])
