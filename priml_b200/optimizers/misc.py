"""AdamATan2, SignSGD and exact-Hessian Newton (``priml/optimizers/adam_atan2.py:33``,
``priml/optimizers/sign_sgd.py:35-349``, ``priml/optimizers/newton.py:18-66``)."""

from __future__ import annotations

from collections.abc import Callable, Iterable
from functools import partial
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor
from torch.optim import Optimizer

from priml_b200.config import Fig

__all__ = ["AdamATan2", "Newton", "SignSGD"]


class AdamATan2(Optimizer):
    """Adam with ``atan2(m, sqrt(v_hat))`` in place of ``m / (sqrt(v_hat) + eps)``
    (Everett et al. 2024): scale invariant and epsilon free."""

    class Config(Fig["Callable[..., AdamATan2]"]):
        lr: float = 1e-3
        betas: tuple[float, float] = (0.9, 0.999)
        weight_decay: float = 1e-2

        def make(self) -> Callable[..., AdamATan2]:
            f = self.copy_tree().finalize()
            return partial(AdamATan2, lr=f.lr, betas=f.betas, weight_decay=f.weight_decay)

    def __init__(self, params: Iterable[Any], lr: float = 1e-3, *, betas: tuple[float, float] = (0.9, 0.999),
                 weight_decay: float = 1e-2) -> None:  # fmt: skip
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}.")
        if any(b < 0.0 or b >= 1.0 for b in betas):
            raise ValueError(f"Invalid betas: {betas}.")
        super().__init__(params, {"lr": lr, "betas": betas, "weight_decay": weight_decay})

    @torch.no_grad()
    def step(self, closure: Callable[[], Any] | None = None) -> Any:
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            b1, b2 = g["betas"]
            lr, wd = g["lr"], g["weight_decay"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    # Plain int step: keeping it a host integer avoids a device sync per parameter.
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p)
                    st["exp_avg_sq"] = torch.zeros_like(p)
                st["step"] += 1
                m, v = st["exp_avg"], st["exp_avg_sq"]
                m.mul_(b1).add_(p.grad, alpha=1.0 - b1)
                v.mul_(b2).addcmul_(p.grad, p.grad, value=1.0 - b2)
                if wd != 0:
                    p.mul_(1.0 - lr * wd)
                step_size = lr / (1.0 - b1 ** st["step"])
                p.add_(torch.atan2(m, v.sqrt() / (1.0 - b2 ** st["step"]) ** 0.5), alpha=-step_size)
        return loss


def _distributed() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


class SignSGD(Optimizer):
    """``p -= lr * sign(g)`` with decay applied only to rows the gradient touched.

    With ``aggregate_distributed`` and more than one rank, rank-local gradient
    rows are all-gathered and summed before the sign (the reference's sparse
    distributed path, ``priml/optimizers/sign_sgd.py:220-349``).

    A group flagged ``{"sparse_embedding": True}`` holds exactly three tensors
    of a sparse embedding: the full ``[N, D]`` table (a buffer), the ``[B, D]``
    gradient leaf holding the batch's rows, and the ``[B]`` row ids. Only the
    rows named by the ids (summed over duplicates and, when aggregating, over
    ranks) are read, decayed and written back; the table never has a dense
    gradient (``priml/optimizers/sign_sgd.py:98-134``).
    """

    class Config(Fig["Callable[..., SignSGD]"]):
        lr: float = 1e-2
        weight_decay: float = 0.0
        aggregate_distributed: bool = True

        def make(self) -> Callable[..., SignSGD]:
            f = self.copy_tree().finalize()
            return partial(SignSGD, lr=f.lr, weight_decay=f.weight_decay, aggregate_distributed=f.aggregate_distributed)

    def __init__(self, params: Iterable[Any], lr: float = 1e-2, *, weight_decay: float = 0.0,
                 aggregate_distributed: bool = True) -> None:  # fmt: skip
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}.")
        super().__init__(params, {"lr": lr, "weight_decay": weight_decay})
        self.aggregate_distributed = aggregate_distributed

    @torch.no_grad()
    def step(self, closure: Callable[[], Any] | None = None) -> Any:
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            lr, wd = g["lr"], g["weight_decay"]
            if g.get("sparse_embedding", False):
                grad, ids, table = _sparse_parts(g["params"])
                if grad is not None:
                    _sparse_row_step(grad, ids, table, lr=lr, weight_decay=wd, aggregate=self.aggregate_distributed)
                continue
            for p in g["params"]:
                grad = p.grad
                if grad is None:
                    continue
                if self.aggregate_distributed and _distributed() and p.ndim >= 2:
                    grad = _gather_row_sum(grad)
                if wd != 0.0:
                    if p.ndim >= 2:
                        touched = grad.reshape(grad.shape[0], -1).any(dim=-1)
                        p.mul_(touched.to(p.dtype).mul_(-lr * wd).add_(1.0).view(-1, *([1] * (p.ndim - 1))))
                    else:
                        p.mul_(1.0 - lr * wd)
                p.add_(torch.sign(grad), alpha=-lr)
        return loss


    @torch.no_grad()
    def step_sparse_embedding(self, rows_grad: Tensor, row_ids: Tensor) -> None:
        """Apply an explicit ``[B, D]`` row gradient for ``row_ids`` to every sparse-embedding group's table."""
        for g in self.param_groups:
            if g.get("sparse_embedding", False):
                _, _, table = _sparse_parts(g["params"])
                _sparse_row_step(rows_grad, row_ids, table, lr=g["lr"], weight_decay=g["weight_decay"],
                                 aggregate=self.aggregate_distributed)  # fmt: skip


def _sparse_parts(params: list[Tensor]) -> tuple[Tensor | None, Tensor, Tensor]:
    """``(leaf.grad, ids, table)`` of a sparse-embedding group, told apart by role, not position."""
    leaf = [p for p in params if p.requires_grad]
    ids = [p for p in params if not p.requires_grad and p.ndim == 1]
    table = [p for p in params if not p.requires_grad and p.ndim == 2]
    if len(params) != 3 or len(leaf) != 1 or len(ids) != 1 or len(table) != 1:
        raise ValueError("a sparse_embedding group holds [table (2-D), rows leaf (2-D, requires_grad), ids (1-D)].")
    return leaf[0].grad, ids[0], table[0]


def _sparse_row_step(rows_grad: Tensor, row_ids: Tensor, table: Tensor, *, lr: float, weight_decay: float,
                     aggregate: bool) -> None:  # fmt: skip
    if aggregate and _distributed():
        world = dist.get_world_size()
        all_rows = rows_grad.new_empty(world * rows_grad.shape[0], rows_grad.shape[1])
        all_ids = row_ids.new_empty(world * row_ids.shape[0])
        dist.all_gather_into_tensor(all_rows, rows_grad.contiguous())
        dist.all_gather_into_tensor(all_ids, row_ids.contiguous())
        rows_grad, row_ids = all_rows, all_ids
    uniq, slot = torch.unique(row_ids.long(), return_inverse=True)
    summed = rows_grad.new_zeros(uniq.numel(), rows_grad.shape[1]).index_add_(0, slot, rows_grad)
    rows = table.index_select(0, uniq)
    if weight_decay != 0.0:
        rows.mul_(1.0 - lr * weight_decay)
    rows.add_(torch.sign(summed).to(rows.dtype), alpha=-lr)
    table.index_copy_(0, uniq, rows)


def _gather_row_sum(grad: Tensor) -> Tensor:
    """Sum of every rank's touched gradient rows (rows + ids all-gathered)."""
    flat = grad.reshape(grad.shape[0], -1)
    ids = flat.any(dim=-1).nonzero().squeeze(-1)
    n = torch.tensor([ids.numel()], device=grad.device)
    world = dist.get_world_size()
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n)
    m = int(max(int(c) for c in counts))
    rows = torch.zeros(m, flat.shape[1], dtype=flat.dtype, device=flat.device)
    idp = torch.full((m,), -1, dtype=torch.int64, device=flat.device)
    rows[: ids.numel()] = flat[ids]
    idp[: ids.numel()] = ids
    all_rows = torch.empty(world * m, flat.shape[1], dtype=flat.dtype, device=flat.device)
    all_ids = torch.empty(world * m, dtype=torch.int64, device=flat.device)
    dist.all_gather_into_tensor(all_rows, rows)
    dist.all_gather_into_tensor(all_ids, idp)
    keep = all_ids >= 0
    out = torch.zeros_like(flat)
    out.index_add_(0, all_ids[keep], all_rows[keep])
    return out.view_as(grad)


class Newton(Optimizer):
    """Exact-Hessian Newton step on a small parameter vector: ``p -= lr * H^-1 g``
    with Levenberg damping; needs a closure returning a graph-bearing loss."""

    requires_closure = True

    class Config(Fig["Callable[..., Newton]"]):
        lr: float = 1.0
        damping: float = 1e-4

        def make(self) -> Callable[..., Newton]:
            f = self.copy_tree().finalize()
            return partial(Newton, lr=f.lr, damping=f.damping)

    def __init__(self, params: Iterable[Any], lr: float = 1.0, *, damping: float = 1e-4) -> None:
        super().__init__(params, {"lr": lr, "damping": damping})

    def step(self, closure: Callable[[], Tensor] | None = None) -> Any:  # type: ignore[override]
        if closure is None:
            raise ValueError("Newton requires a closure returning the loss.")
        params = [p for g in self.param_groups for p in g["params"] if p.requires_grad]
        with torch.enable_grad():
            loss = closure()
            grads = torch.autograd.grad(loss, params, create_graph=True)
            flat = torch.cat([g.reshape(-1) for g in grads])
            rows = [torch.cat([h.reshape(-1) for h in torch.autograd.grad(flat[i], params, retain_graph=True)])
                    for i in range(flat.numel())]  # fmt: skip
        hess = torch.stack(rows).detach()
        g0 = self.param_groups[0]
        hess = hess + g0["damping"] * torch.eye(hess.shape[0], dtype=hess.dtype, device=hess.device)
        step = torch.linalg.solve(hess, flat.detach())
        with torch.no_grad():
            off = 0
            for p in params:
                n = p.numel()
                p.sub_(g0["lr"] * step[off : off + n].view_as(p))
                off += n
        return loss
