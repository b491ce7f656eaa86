"""The training run (``priml/train/train_loop.py:206-1581``).

``TrainLoop(config).run()``: runtime init -> seeding (model seed salted by the
``pp`` coordinate, data seed by ``dp``) -> build step, dataset, metrics,
checkpointer, tracker -> resume (+ overwrite guard) -> loop:

    batch fetch (host->device) -> epoch tick -> cadence save / eval ->
    train_step -> periodic logging (one all_reduce of the metric vector and
    one device->host read per log interval) -> time-limit check

Stop decisions that depend on clocks are made on rank 0 and broadcast, so
ranks never disagree on whether to take another collective step. The run ends
with a final save, a final eval and a ``RESULT:`` line.
"""

from __future__ import annotations

import gc
import logging
import math
import time
from dataclasses import field
from pathlib import Path
from typing import Any, Literal

import torch
import torch.distributed as dist

from priml_b200.config import Fig
from priml_b200.data import DummyDataset
from priml_b200.math.seed import get_rng_state, salt, set_rng_state, set_seed_distributed, set_seed_local
from priml_b200.parallel.runtime import SingleProcess, global_device_mesh, is_rank_zero
from priml_b200.train.train_step import TrainStep

__all__ = ["EvalTimeLimitError", "TrainLoop"]

log = logging.getLogger(__name__)


class EvalTimeLimitError(RuntimeError):
    """Eval exceeded ``max_eval_time`` with ``eval_stop_on_time_limit``."""


def _dist() -> bool:
    return dist.is_available() and dist.is_initialized()


class TrainLoop:
    class Config(Fig["TrainLoop"]):
        study_name: str = ""
        experiment_name: str = ""
        base_dir: Path | str | None = None
        working_dir: Path | str = "runs/{study_name}/{experiment_name}"
        doc: str = ""
        step: Any = field(default_factory=TrainStep.Config)
        dataset: Any = field(default_factory=DummyDataset.Config)
        metrics: dict[str, Any] = field(default_factory=dict)
        checkpointing: Any = None
        profiling: Any = None
        phase_timer: Any = None
        tracker: Any = None
        max_steps: float = math.inf
        max_epochs: float = math.inf
        max_time: float = math.inf
        max_time_kind: Literal["wall", "train"] = "wall"
        max_eval_time: float = math.inf
        eval_stop_on_time_limit: bool = False
        num_steps_eval: float = 1_000
        num_steps_log: int = 10
        early_train_log_steps: int = 100
        phase_heartbeat_sec: float = 20.0
        eval_every_epoch: bool = True
        eval_warmup_batches: int = 0
        eval_only: bool = False
        restore_rng_state: bool = True
        seed: int | None = None
        num_steps_garbage_collect: float = math.inf
        mesh_dim_model_seed: str = "pp"
        mesh_dim_data_seed: str = "dp"
        runtime: Any = field(default_factory=SingleProcess.Config)

        def finalize(self):  # noqa: ANN201
            if not math.isfinite(self.max_steps) and math.isfinite(getattr(self.step, "train_budget_steps", math.inf)):
                self.max_steps = self.step.train_budget_steps
            if self.checkpointing is not None and getattr(self.checkpointing, "base_dir", None) is None:
                self.checkpointing.base_dir = str(self.resolved_working_dir())
            return super().finalize()

        def resolved_working_dir(self) -> Path:
            wd = str(self.working_dir).format(study_name=self.study_name, experiment_name=self.experiment_name or "run")
            base = Path(self.base_dir) if self.base_dir is not None else Path(".")
            p = Path(wd)
            return p if p.is_absolute() else base / p

    def __init__(self, config: Config) -> None:
        self.config = config
        self.runtime = config.runtime.make()
        self.runtime.initialize()
        try:
            self._build()
        except BaseException:
            self.runtime.destroy()
            raise

    def _axis_coord(self, name: str) -> int:
        mesh = global_device_mesh()
        if mesh is None or name not in (mesh.mesh_dim_names or ()):
            return 0
        return mesh[name].get_local_rank()

    def _build(self) -> None:
        c = self.config
        if _dist():
            seed = set_seed_distributed(c.seed, axis_salts=("model", self._axis_coord(c.mesh_dim_model_seed)))
        else:
            seed = set_seed_local(c.seed if c.seed is not None else 0)
        self.seed = seed
        self.step = c.step.make()
        self.metrics = {k: v.make() for k, v in c.metrics.items()}
        set_seed_local((seed + salt("data", self._axis_coord(c.mesh_dim_data_seed))) % (2**63) or 1)
        self.dataset = c.dataset.make()
        self.step.bind_epoch_timer(getattr(self.dataset, "timer_epoch", None))
        if hasattr(self.dataset, "bind_step"):  # datasets that serve the learner's own policy (RL)
            self.dataset.bind_step(self.step)
        self.checkpointing = c.checkpointing.make() if c.checkpointing is not None else None
        self.tracker = c.tracker.make() if c.tracker is not None else None
        self.profiling = c.profiling.make() if c.profiling is not None else None
        self.phase_timer = c.phase_timer.make() if c.phase_timer is not None else None
        self.global_step = 0
        self.epoch = 0
        self.train_seconds = 0.0
        self.eval_seconds = 0.0
        self.last_eval: dict[str, float] = {}
        self._t_start = time.perf_counter()
        if _dist():
            dist.barrier()
        if self.checkpointing is not None:
            resumed = self.checkpointing.load(self, max_steps=c.max_steps, guard=True)
            if resumed is not None:
                log.info("resumed from step %d", resumed)

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict[str, Any]:
        return {
            "step": self.step.state_dict(),
            "dataset": self.dataset.state_dict() if hasattr(self.dataset, "state_dict") else {},
            "metrics": {k: m.state_dict() for k, m in self.metrics.items() if hasattr(m, "state_dict")},
            "rng": get_rng_state(),
        }

    def load_state_dict(self, s: dict[str, Any]) -> None:
        self.step.load_state_dict(s["step"])
        if hasattr(self.dataset, "load_state_dict"):
            self.dataset.load_state_dict(s.get("dataset", {}))
        for k, m in self.metrics.items():
            if k in s.get("metrics", {}) and hasattr(m, "load_state_dict"):
                m.load_state_dict(s["metrics"][k])
        if self.config.restore_rng_state and "rng" in s:
            set_rng_state(s["rng"])
        # Progress is not stored twice: optimizer steps ride the step's timer and completed
        # passes the dataset's epoch timer, as in the reference's checkpoints.
        self.global_step = int(getattr(self.step, "global_step", self.step.timer_step.global_count))
        epochs = getattr(self.dataset, "timer_epoch", None)
        self.epoch = int(epochs.global_count) if epochs is not None else 0

    # ------------------------------------------------------------------ helpers
    def _time_limit_reached(self) -> bool:
        c = self.config
        if not math.isfinite(c.max_time):
            return False
        used = time.perf_counter() - self._t_start if c.max_time_kind == "wall" else self._train_elapsed()
        hit = used >= c.max_time
        if _dist():
            dev = self.step.device if self.step.device.type == "cuda" else torch.device("cpu")
            t = torch.tensor([1.0 if hit else 0.0], device=dev)
            dist.broadcast(t, src=0)
            hit = bool(t.item() > 0)
        return hit

    def _log(self, out: dict[str, Any], dt: float) -> None:
        keys = sorted(k for k, v in out.items() if isinstance(v, torch.Tensor) and k != "model" and v.is_floating_point())
        vals = torch.stack([out[k].detach().float().mean() for k in keys])
        if _dist():
            dist.all_reduce(vals)
            vals = vals / dist.get_world_size()
        host = vals.tolist()
        rec = {f"train/{'total_loss' if k == 'loss' else k}": v for k, v in zip(keys, host, strict=True)}
        rec["step_time"] = dt
        rec["elapsed"] = time.perf_counter() - self._t_start
        if torch.cuda.is_available():
            rec["gpu_mem_alloc_gb"] = torch.cuda.memory_allocated() / 1e9
            rec["gpu_mem_peak_gb"] = torch.cuda.max_memory_allocated() / 1e9
        if is_rank_zero():
            log.info("Step %d/%s: loss=%.4f step_time=%.3fs", self.global_step, self.config.max_steps,
                     rec.get("train/total_loss", float("nan")), dt)  # fmt: skip
        if self.tracker is not None:
            self.tracker.log(rec, self.global_step)
        self.last_log = rec

    # ------------------------------------------------------------------ eval
    @torch.no_grad()
    def eval(self) -> dict[str, float]:
        t0 = time.perf_counter()
        total, n = None, 0
        for m in self.metrics.values():
            m.reset()
        for i, batch in enumerate(self.dataset.eval_dataloader()):
            batch = self.step.preprocess_batch(batch)
            out = self.step.eval_loss(**batch)
            if i < self.config.eval_warmup_batches:
                continue
            for m in self.metrics.values():
                m.update(out.get("model"), **batch)
            v = out["loss"].float().mean()
            total = v if total is None else total + v
            n += 1
            if time.perf_counter() - t0 > self.config.max_eval_time:
                if self.config.eval_stop_on_time_limit:
                    raise EvalTimeLimitError(f"eval exceeded {self.config.max_eval_time}s")
                break
        res: dict[str, float] = {}
        if total is not None:
            t = total / n
            if _dist():
                dist.all_reduce(t)
                t = t / dist.get_world_size()
            res["eval/total_loss"] = float(t)
        for k, m in self.metrics.items():
            for key, value in m.compute().items():
                res[f"eval/{k}_{key}" if k else f"eval/{key}"] = float(value)
        self.eval_seconds += time.perf_counter() - t0
        if self.tracker is not None and res:
            self.tracker.log(res, self.global_step)
        self.last_eval = res
        return res

    def _maybe_eval(self, *, is_final: bool = False) -> None:
        c = self.config
        due = is_final or (math.isfinite(c.num_steps_eval) and c.num_steps_eval > 0 and self.global_step > 0
                           and self.global_step % int(c.num_steps_eval) == 0)  # <= 0: only the final eval
        if due:
            self.eval()

    # ------------------------------------------------------------------ main
    def run(self, *args: Any) -> dict[str, float]:
        del args
        try:
            if self.config.eval_only:
                return self.eval()
            return self.train()
        finally:
            self._cleanup()

    def _train_elapsed(self) -> float:
        """Seconds the ``train`` time limit counts (a step with its own budget clock overrides this)."""
        return self.train_seconds

    def _on_batch_ready(self, fetch_time: float) -> None:
        """Called with the seconds spent fetching each training batch (no-op by default)."""
        del fetch_time

    def train(self) -> dict[str, float]:
        c = self.config
        it = iter(self.dataset.train_dataloader())
        window_t0 = time.perf_counter()
        while self.global_step < c.max_steps and self.epoch < c.max_epochs:
            try:
                fetch_t0 = time.perf_counter()
                batch = next(it)
                self._on_batch_ready(time.perf_counter() - fetch_t0)
            except StopIteration:
                self.epoch += 1
                passes = getattr(self.dataset, "timer_epoch", None)
                if passes is not None:  # the dataset checkpoints its pass count
                    passes.global_count += 1
                    passes.local_count += 1
                self.step.on_epoch_end()
                if c.eval_every_epoch and self.metrics:
                    self.eval()
                if self.epoch >= c.max_epochs:
                    break
                it = iter(self.dataset.train_dataloader())
                continue
            if self.profiling is not None:
                self.profiling.on_step_start(self.global_step)
            t0 = time.perf_counter()
            batch = self.step.preprocess_batch(batch)
            out = self.step.train_step(**batch)
            if out.get("stepped", True):
                self.global_step += 1
            self.train_seconds += time.perf_counter() - t0
            if self.profiling is not None:
                self.profiling.on_step_end(self.global_step)
            if self.checkpointing is not None:
                self.checkpointing.maybe_save(self, self.global_step)
            self._maybe_eval()
            early = self.global_step <= c.early_train_log_steps and self.global_step % max(1, c.num_steps_log // 10 or 1) == 0
            if self.global_step % max(1, c.num_steps_log) == 0 or early:
                now = time.perf_counter()
                self._log(dict(out), now - window_t0)
                window_t0 = now
                if self._time_limit_reached():
                    break
            if math.isfinite(c.num_steps_garbage_collect) and self.global_step % int(c.num_steps_garbage_collect) == 0:
                gc.collect()
        if self.checkpointing is not None:
            self.checkpointing.save(self, self.global_step)
            self.checkpointing.flush()
        self._maybe_eval(is_final=True)
        if is_rank_zero():
            wall = time.perf_counter() - self._t_start
            log.info("RESULT: steps=%d train=%.1fs eval=%.1fs other=%.1fs %s", self.global_step, self.train_seconds,
                     self.eval_seconds, wall - self.train_seconds - self.eval_seconds, self.last_eval)  # fmt: skip
        return self.last_eval

    def _cleanup(self) -> None:
        if self.tracker is not None:
            self.tracker.flush()
            self.tracker.close()
        if self.phase_timer is not None:
            self.phase_timer.close()
        self.runtime.destroy()
