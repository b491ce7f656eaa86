"""AdamW with a single fused step (``priml/optimizers/fused_adamw.py:42-244``).

Arithmetic order is the reference's: ``p *= 1 - lr*wd``; ``m = lerp(m, g, 1-b1)``;
``v = lerp(v, g^2, 1-b2)``; ``p -= m / (sqrt(v / bias2) + eps) * (lr / bias1)``.

On CUDA every parameter of every group is updated by ONE multi-tensor kernel
launch per group (``priml_b200.ops._C.MultiTensorPlan``): device-resident
pointer tables built once, 64K-element chunks, and -- when a parameter has a
bf16 compute shadow -- the refreshed shadow written in the same pass. Optional
global-norm clipping is folded in as a device-side scale (no host sync).
State keys match the reference: ``step``, ``first_moment``, ``second_moment``.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable
from functools import partial
from typing import Any

import torch
from torch import Tensor
from torch.optim import Optimizer

from priml_b200 import ops
from priml_b200.config import Fig

__all__ = ["FusedAdamW"]


def _local(t: Tensor) -> Tensor:
    """The rank-local shard of a DTensor (FSDP2 / TP parameter), else ``t``."""
    return t._local_tensor if hasattr(t, "_local_tensor") else t  # noqa: SLF001


class FusedAdamW(Optimizer):
    class Config(Fig["Callable[..., FusedAdamW]"]):
        lr: float = 1e-3
        betas: tuple[float, float] = (0.9, 0.999)
        eps: float = 1e-8
        weight_decay: float = 0.0
        compile: bool = True
        """Kept for config compatibility; the CUDA path is always one fused kernel."""

        def make(self) -> Callable[..., FusedAdamW]:
            f = self.copy_tree().finalize()
            return partial(FusedAdamW, lr=f.lr, betas=f.betas, eps=f.eps, weight_decay=f.weight_decay, compile=f.compile)

    def __init__(
        self,
        params: Iterable[Tensor] | Iterable[dict[str, Any]],
        lr: float = 1e-3,
        *,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.0,
        compile: bool = True,  # noqa: A002
    ) -> None:
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}.")
        if not all(0.0 <= b < 1.0 for b in betas):
            raise ValueError(f"betas must lie in [0, 1); got {betas}.")
        if eps < 0.0:
            raise ValueError(f"Invalid eps: {eps}.")
        if weight_decay < 0.0:
            raise ValueError(f"Invalid weight_decay: {weight_decay}.")
        super().__init__(params, {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay})
        self.compile = compile
        self._plans: dict[int, tuple[Any, ...]] = {}
        self.grad_scale: Tensor | None = None
        """Optional fp32 device scalar multiplying every gradient (clip coefficient)."""

    # ------------------------------------------------------------------ helpers
    def _state(self, p: Tensor) -> dict[str, Any]:
        st = self.state[p]
        if not st:
            st["step"] = 0
            st["first_moment"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            st["second_moment"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        return st

    def _plan(self, gi: int, params: list[Tensor]) -> Any:
        """Cached device tensor table for group ``gi`` (rebuilt when any pointer moves)."""
        if not params or not ops.native_available() or ops.reference_forced():
            return None
        lp = [_local(p) for p in params]
        if any(p.dtype != torch.float32 or not p.is_contiguous() or not p.is_cuda for p in lp):
            return None
        grads = [_local(p.grad) if p.grad is not None else None for p in params]
        if any(g is None or not g.is_contiguous() or g.dtype not in (torch.float32, torch.bfloat16) for g in grads):
            return None
        states = [self._state(p) for p in params]
        ms = [_local(st["first_moment"]) for st in states]
        vs = [_local(st["second_moment"]) for st in states]
        shadows = []
        for p in params:
            cached = getattr(_local(p), "_pb_shadow", None) or getattr(p, "_pb_shadow", None)
            shadows.append(cached[1] if cached is not None and cached[1].is_contiguous() else None)
        key = tuple(
            (p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), None if s is None else s.data_ptr(), g.dtype)
            for p, g, m, v, s in zip(lp, grads, ms, vs, shadows, strict=True)
        )
        plan = self._plans.get(gi)
        if plan is None or plan[0] != key:
            plan = (key, ops.native().MultiTensorPlan([p.detach() for p in lp], grads, ms, vs, shadows, 65536), shadows)
            self._plans[gi] = plan
        return plan

    def fused_grad_norm(self, max_norm: float) -> tuple[Tensor, Tensor] | None:
        """Global gradient norm and clip coefficient as device scalars (no host sync)."""
        sq = None
        sharded = False
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            plan = self._plan(gi, params)
            if plan is None:
                return None
            sharded = sharded or any(hasattr(p, "_local_tensor") for p in params)
            n, _ = plan[1].grad_norm_clip(1.0)
            sq = n * n if sq is None else sq + n * n
        if sq is None:
            return None
        if sharded and torch.distributed.is_available() and torch.distributed.is_initialized():
            torch.distributed.all_reduce(sq)
        norm = sq.sqrt()
        return norm, (max_norm / (norm + 1e-6)).clamp(max=1.0)

    def _native_group(self, gi: int, group: dict[str, Any], params: list[Tensor]) -> bool:
        from priml_b200.ops import functional as fn

        plan = self._plan(gi, params)
        if plan is None:
            return False
        states = [self._state(p) for p in params]
        steps = {st["step"] for st in states}
        if len(steps) != 1:
            return False
        shadows = plan[2]
        step = next(iter(steps)) + 1
        for st in states:
            st["step"] = step
        b1, b2 = group["betas"]
        t = torch.tensor([b1, b2], dtype=torch.float32)
        bias1 = float(1 - t[0] ** step)
        bias2 = float(1 - t[1] ** step)
        plan[1].adamw(group["lr"], b1, b2, group["eps"], group["weight_decay"], bias1, bias2, self.grad_scale)
        for p, s in zip(params, shadows, strict=True):
            if s is not None:
                fn.mark_shadow_fresh(_local(p))
            else:
                fn.forget_quantized(_local(p))
            fn.forget_quantized(p)
        return True

    @torch.no_grad()
    def step(self, closure: Callable[[], Any] | None = None) -> Any:
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            if params[0].is_cuda and self._native_group(gi, group, params):
                continue
            b1, b2 = group["betas"]
            for p in params:
                st = self._state(p)
                st["step"] += 1
                g = p.grad if self.grad_scale is None else p.grad * self.grad_scale.to(p.grad.device)
                ops.reference.adamw_(
                    [p.data], [g], [st["first_moment"]], [st["second_moment"]],
                    step=st["step"], lr=group["lr"], beta1=b1, beta2=b2, eps=group["eps"],
                    weight_decay=group["weight_decay"],
                )  # fmt: skip
        return loss

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        super().load_state_dict(state_dict)
        self._plans.clear()
