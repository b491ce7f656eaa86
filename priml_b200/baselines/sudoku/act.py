"""Adaptive computation time over a fixed pool of puzzle slots (``priml/baselines/sudoku/act.py:1-375``).

The pool holds ``batch_size`` slots; each train step every slot takes ONE
recurrent step from its carried latents. A slot that halted last step is
re-seated with the incoming batch's puzzle (fresh zero latents, step count 0);
the others keep theirs. So the batch shape never changes, easy puzzles leave
early and hard ones keep their slot -- with no host round trip: seating,
feedback and halting are ``torch.where`` selections on device tensors.

Halting: a slot halts when its halt logit is positive (after a minimum step
count) or when it reaches ``max_steps``. With probability
``halt_exploration_prob`` a slot draws its minimum from ``[2, max_steps]``
(``min_steps_sampled``) -- the counterfactual a self-supervised halt head
never sees otherwise. The draws come from a dedicated generator so the training
trajectory does not depend on ambient RNG state.

The halt head is trained with binary cross-entropy against "every counted
cell is right", weighted by ``halt_weight``.
"""

from __future__ import annotations

from typing import TYPE_CHECKING, Any

import torch
from torch import Tensor, nn

from priml_b200.config import Fig

if TYPE_CHECKING:
    from priml_b200.baselines.sudoku.model import SudokuNet

__all__ = ["ActPool"]


class ActPool:
    class Config(Fig["ActPool"]):
        batch_size: int = 384
        max_steps: int = 32
        halt_weight: float = 0.05
        halt_exploration_prob: float = 0.1
        halt_exploration_seed: int = 0
        min_steps_sampled: bool = True
        feedback: bool = True
        """Feed the decoded grid (givens restored) back as the next step's feedback channel."""
        given_low: int = 2
        given_high: int = 10
        """Tokens in ``[given_low, given_high]`` are clues and are never overwritten in the feedback."""
        grid_len: int = -1
        seq_len: int = -1
        hidden_size: int = -1

        def finalize(self):  # noqa: ANN201
            if self.given_low > self.given_high:
                raise ValueError(f"given_low {self.given_low} exceeds given_high {self.given_high}.")
            return super().finalize()

    def __init__(self, config: Config) -> None:
        if min(config.grid_len, config.seq_len, config.hidden_size) <= 0:
            raise ValueError(
                "grid_len, seq_len and hidden_size must be positive (inherited from the model); got "
                f"{config.grid_len}, {config.seq_len}, {config.hidden_size}."
            )
        self.config = config
        self.device = torch.device("cpu")
        n = config.batch_size
        self.inputs = torch.zeros(n, config.grid_len, dtype=torch.long)
        self.labels = torch.zeros_like(self.inputs)
        self.feedback = torch.zeros_like(self.inputs)
        self.z_slow = torch.zeros(n, config.seq_len, config.hidden_size)
        self.z_fast = torch.zeros_like(self.z_slow)
        self.steps = torch.zeros(n, dtype=torch.long)
        self.halted = torch.ones(n, dtype=torch.bool)
        self.identifiers = torch.zeros(n, dtype=torch.long)
        self._generator = self._new_generator()

    def _new_generator(self) -> torch.Generator:
        g = torch.Generator(device=self.device)
        g.manual_seed(self.config.halt_exploration_seed)
        return g

    def to(self, device: torch.device | str) -> None:
        self.device = torch.device(device)
        for name in ("inputs", "labels", "feedback", "z_slow", "z_fast", "steps", "halted", "identifiers"):
            setattr(self, name, getattr(self, name).to(self.device))
        self._generator = self._new_generator()

    def latents(self) -> tuple[Tensor, Tensor]:
        return self.z_slow, self.z_fast

    def refill(self, media: Tensor, *, labels: Tensor, valid_count: int, ignore_label_id: int,
               identifiers: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:  # fmt: skip
        """Seat the incoming batch in halted slots; returns ``(inputs, labels, active)``.

        Per-puzzle ``identifiers`` are seated alongside, so a slot that keeps its
        puzzle also keeps that puzzle's prefix row (:attr:`identifiers`).
        """
        n = self.config.batch_size
        if media.shape[0] != n:
            raise ValueError(f"the pool holds {n} slots; got a batch of {media.shape[0]}.")
        new_labels = labels.to(torch.long).clone()
        if valid_count < n:
            new_labels[valid_count:] = ignore_label_id
        seat = self.halted[:, None]
        self.inputs = torch.where(seat, media.to(torch.long), self.inputs)
        self.labels = torch.where(seat, new_labels, self.labels)
        self.steps = self.steps.masked_fill(self.halted, 0)
        seat3 = self.halted[:, None, None]
        self.z_slow = self.z_slow.masked_fill(seat3, 0.0)
        self.z_fast = self.z_fast.masked_fill(seat3, 0.0)
        self.feedback = torch.where(seat, self.inputs, self.feedback)
        if identifiers is not None:
            self.identifiers = torch.where(self.halted, identifiers.to(torch.long), self.identifiers)
        return self.inputs, self.labels, torch.ones_like(self.halted)

    def advance(self, z_slow: Tensor, *, z_fast: Tensor, logits: Tensor, halt: Tensor, media: Tensor) -> None:
        """Store the step's latents, decoded feedback and halting decision."""
        self.z_slow = z_slow.to(self.z_slow.dtype)
        self.z_fast = z_fast.to(self.z_fast.dtype)
        self.steps = self.steps + 1
        if self.config.feedback:
            self.feedback = self.clamp_givens(logits.detach().argmax(dim=-1), media=media)
        self.halted = self._halt_mask(halt)

    def rollout(self, model: SudokuNet, *, media: Tensor,
                prefix_kwargs: dict[str, Any] | None = None) -> tuple[Tensor, Tensor]:  # fmt: skip
        """Evaluation: every example runs exactly ``max_steps`` steps; returns the last logits and halt."""
        z_slow, z_fast = model.init_latents(media.shape[0])
        feedback = media if self.config.feedback else None
        logits = halt = None
        for _ in range(self.config.max_steps):
            self.set_feedback(model, feedback)
            out = model(media, z_slow, z_fast, **(prefix_kwargs or {}))
            z_slow, z_fast, logits, halt = out.z_slow, out.z_fast, out.logits, out.halt
            if feedback is not None:
                feedback = self.clamp_givens(logits.argmax(dim=-1), media=media)
        assert logits is not None and halt is not None
        return logits, halt

    def halt_loss(self, logits: Tensor, *, labels: Tensor, halt: Tensor, active: Tensor,
                  ignore_label_id: int) -> tuple[Tensor, dict[str, Any]]:  # fmt: skip
        with torch.no_grad():
            counted = labels != ignore_label_id
            right = (logits.argmax(dim=-1) == labels) & counted
            per_row = counted.sum(-1)
            solved = ((right.sum(-1) == per_row) & (per_row > 0)).to(halt.dtype)
        per = nn.functional.binary_cross_entropy_with_logits(halt, solved, reduction="none")
        loss = (per * active).sum() / active.sum().clamp(min=1)
        metrics = {"halt_loss": loss.detach(), "halted_frac": self.halted.float().mean(),
                   "act_steps": self.steps.float().mean()}  # fmt: skip
        return self.config.halt_weight * loss, metrics

    def clamp_givens(self, decoded: Tensor, *, media: Tensor) -> Tensor:
        given = (media >= self.config.given_low) & (media <= self.config.given_high)
        return torch.where(given, media.to(decoded.dtype), decoded)

    @staticmethod
    def set_feedback(model: SudokuNet, feedback: Tensor | None) -> None:
        if feedback is None:
            return
        for ch in model.embedding.channels:
            setter = getattr(ch, "set_feedback", None)
            if setter is not None:
                setter(feedback)

    def _halt_mask(self, halt: Tensor) -> Tensor:
        c = self.config
        n = c.batch_size
        at_cap = self.steps >= c.max_steps
        fired = halt > 0
        explore = torch.rand(n, device=self.device, generator=self._generator) < c.halt_exploration_prob
        if c.min_steps_sampled:
            sampled = torch.randint(2, c.max_steps + 1, (n,), device=self.device, generator=self._generator)
            minimum = torch.where(explore, sampled, torch.ones_like(sampled))
            return at_cap | (fired & (self.steps >= minimum))
        return at_cap | (fired & ~explore)

    def state_dict(self) -> dict[str, Any]:
        return {"halt_rng": self._generator.get_state()}

    def load_state_dict(self, s: dict[str, Any]) -> None:
        if "halt_rng" in s:
            self._generator.set_state(s["halt_rng"].cpu())
