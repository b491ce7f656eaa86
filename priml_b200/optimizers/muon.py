"""Muon and NorMuon (``priml/optimizers/muon.py:38-253``, ``priml/optimizers/normuon.py:55-407``).

Both orthogonalize a momentum update with a bf16 polynomial iteration whose
matmuls run on the tensor cores as plain batched library GEMMs (``@`` on stacked
``[N, R, C]`` buckets: one launch per product for the whole bucket).
NorMuon stacks same-shape parameters and adds a per-row second-moment rescale
and "cautious" weight decay. State keys match the reference (``momentum_buffer``;
NorMuon keeps ``momentum_buffer`` / ``second_moment`` on the first parameter of
each shape bucket).
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterable
from functools import partial
from typing import Any

import torch
from torch import Tensor
from torch.nn import Parameter
from torch.optim import Optimizer

from priml_b200.config import Fig
from priml_b200.math.numeric import POLAR_EXPRESS_COEFFICIENTS, matrix_signum_via_newtonschulz, polar_express

__all__ = [
    "Muon",
    "NorMuon",
    "adjust_lr_conv_heuristic",
    "adjust_lr_match_rms_adamw",
    "adjust_lr_original",
]


def _shape(p: Tensor, ensemble_dims: int) -> tuple[int, int]:
    s = p.shape[ensemble_dims:]
    return int(s[0]), int(math.prod(s[1:]))


def adjust_lr_original(lr: float, param: Tensor, ensemble_dims: int = 0) -> float:
    """``lr * sqrt(max(1, fan_out / fan_in))`` (K. Jordan)."""
    c_out, c_in = _shape(param, ensemble_dims)
    return lr * math.sqrt(max(1, c_out / c_in))


def adjust_lr_match_rms_adamw(lr: float, param: Tensor, ensemble_dims: int = 0) -> float:
    c_out, c_in = _shape(param, ensemble_dims)
    return lr * 0.2 * math.sqrt(max(c_out, c_in))


def adjust_lr_conv_heuristic(lr: float, param: Tensor, ensemble_dims: int = 0) -> Tensor:
    c_out, _ = _shape(param, ensemble_dims)
    return lr * param.data.norm() / math.sqrt(c_out)


class Muon(Optimizer):
    """Nesterov momentum -> Newton-Schulz orthogonalization -> shape-scaled step."""

    @classmethod
    def eligible_tensor(cls, name: str, parameter: Parameter) -> bool:
        del cls, name
        return parameter.ndim >= 2

    class Config(Fig["Callable[..., Muon]"]):
        lr: float = 1e-3
        weight_decay: float | None = 0.1
        momentum: float = 0.95
        nesterov: bool = True
        ns_coefficients: tuple[float, float, float] = (3.4445, -4.7750, 2.0315)
        eps: float = 1e-7
        ns_steps: int = 5
        adjust_lr_fn: Callable[..., Any] = adjust_lr_original
        ensemble_dims: int = 0

        def make(self) -> Callable[..., Muon]:
            f = self.copy_tree().finalize()
            return partial(
                Muon, lr=f.lr, weight_decay=f.weight_decay, momentum=f.momentum, nesterov=f.nesterov,
                ns_coefficients=f.ns_coefficients, eps=f.eps, ns_steps=f.ns_steps, adjust_lr_fn=f.adjust_lr_fn,
                ensemble_dims=f.ensemble_dims,
            )  # fmt: skip

    def __init__(
        self,
        params: Iterable[Tensor] | Iterable[dict[str, Any]],
        lr: float = 1e-3,
        *,
        weight_decay: float | None = 0.1,
        momentum: float = 0.95,
        nesterov: bool = True,
        ns_coefficients: tuple[float, float, float] = (3.4445, -4.7750, 2.0315),
        eps: float = 1e-7,
        ns_steps: int = 5,
        adjust_lr_fn: Callable[..., Any] = adjust_lr_original,
        ensemble_dims: int = 0,
    ) -> None:
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if momentum < 0.0:
            raise ValueError(f"Invalid momentum: {momentum}")
        if weight_decay is not None and weight_decay < 0.0:
            raise ValueError(f"Invalid weight_decay: {weight_decay}")
        if nesterov and momentum <= 0:
            raise ValueError("Nesterov momentum requires momentum > 0")
        self.adjust_lr_fn = adjust_lr_fn
        super().__init__(
            params,
            {"lr": lr, "weight_decay": weight_decay, "momentum": momentum, "nesterov": nesterov,
             "ns_coefficients": ns_coefficients, "eps": eps, "ns_steps": ns_steps, "ensemble_dims": ensemble_dims},
        )  # fmt: skip

    @torch.no_grad()
    def step(self, closure: Callable[[], float] | None = None) -> None:  # type: ignore[override]
        del closure
        for group in self.param_groups:
            lr, wd, mom = group["lr"], group["weight_decay"], group["momentum"]
            ed = group["ensemble_dims"]
            for p in group["params"]:
                g = p.grad
                if g is None:
                    continue
                if g.ndim < 2:
                    raise ValueError(f"Muon requires ndim >= 2, got shape {tuple(p.shape)}.")
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(g)
                buf = st["momentum_buffer"]
                buf.lerp_(g, 1 - mom)
                u = g.lerp(buf, mom) if group["nesterov"] else buf
                o = matrix_signum_via_newtonschulz(
                    u.reshape(math.prod(u.shape[:ed]), u.shape[ed], -1),
                    coefficients=group["ns_coefficients"],
                    steps=group["ns_steps"],
                    eps=group["eps"],
                ).reshape(u.shape)
                if wd is not None:
                    p.data.mul_(1 - lr * wd)
                alr = self.adjust_lr_fn(lr, p, ed)
                if isinstance(alr, Tensor):
                    p.data.add_(o * (-alr))
                else:
                    p.data.add_(o, alpha=-alr)


def _normuon_update(
    grads: Tensor, params: Tensor, mbuf: Tensor, second: Tensor, *, momentum: float, lr: float,
    weight_decay: float, beta2: float, ns_steps: int, reduce_dim: int, coefficients: tuple,
) -> None:  # fmt: skip
    """Momentum, Polar-Express orthogonalization, per-row second-moment rescale
    (norm preserving), cautious decoupled decay -- all on stacked ``[N, R, C]``."""
    mbuf.lerp_(grads, 1 - momentum)
    upd = grads.lerp_(mbuf, momentum)
    x = polar_express(upd, steps=ns_steps, coefficients=coefficients)
    energy = x.float().square().mean(dim=reduce_dim, keepdim=True)
    width = x.size(reduce_dim)
    before = (energy.sum(dim=(-2, -1), keepdim=True) * width).sqrt()
    second.lerp_(energy.to(second.dtype), 1 - beta2)
    scale = second.clamp_min(1e-10).rsqrt()
    after = ((energy * width) * scale.float().square()).sum(dim=(-2, -1), keepdim=True).sqrt()
    x = x * (scale * (before / after.clamp_min(1e-10))).to(x.dtype)
    agrees = (x * params) >= 0
    params.sub_(lr * x + lr * weight_decay * params * agrees)


def _by_shape(params: list[Tensor]) -> list[list[Tensor]]:
    buckets: dict[tuple[int, ...], list[Tensor]] = {}
    for p in params:
        if p.grad is not None:
            buckets.setdefault(tuple(p.shape), []).append(p)
    return [buckets[s] for s in sorted(buckets)]


class NorMuon(Optimizer):
    """Muon with a per-row (or per-column, for wide matrices) second moment."""

    @classmethod
    def eligible_tensor(cls, name: str, parameter: Parameter) -> bool:
        del cls, name
        return parameter.ndim >= 2

    class Config(Fig["Callable[..., NorMuon]"]):
        lr: float = 0.04
        momentum: float = 0.95
        beta2: float = 0.95
        ns_steps: int = 5
        weight_decay: float = 0.2
        compile: bool = True
        coefficients: tuple[tuple[float, float, float], ...] = POLAR_EXPRESS_COEFFICIENTS

        def make(self) -> Callable[..., NorMuon]:
            f = self.copy_tree().finalize()
            return partial(
                NorMuon, lr=f.lr, momentum=f.momentum, beta2=f.beta2, ns_steps=f.ns_steps,
                weight_decay=f.weight_decay, compile=f.compile, coefficients=f.coefficients,
            )  # fmt: skip

    def __init__(
        self,
        params: Iterable[Tensor] | Iterable[dict[str, Any]],
        lr: float = 0.04,
        *,
        momentum: float = 0.95,
        beta2: float = 0.95,
        ns_steps: int = 5,
        weight_decay: float = 0.2,
        compile: bool = True,  # noqa: A002
        coefficients: tuple[tuple[float, float, float], ...] = POLAR_EXPRESS_COEFFICIENTS,
    ) -> None:
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}.")
        if not 0.0 <= momentum < 1.0:
            raise ValueError(f"momentum must lie in [0, 1); got {momentum}.")
        if not 0.0 <= beta2 < 1.0:
            raise ValueError(f"beta2 must lie in [0, 1); got {beta2}.")
        if weight_decay < 0.0:
            raise ValueError(f"Invalid weight_decay: {weight_decay}.")
        if not 1 <= ns_steps <= len(coefficients):
            raise ValueError(f"ns_steps must lie in [1, {len(coefficients)}]; got {ns_steps}.")
        super().__init__(
            params,
            {"lr": lr, "momentum": momentum, "beta2": beta2, "ns_steps": ns_steps, "weight_decay": weight_decay,
             "coefficients": coefficients},
        )  # fmt: skip
        self.compile = compile

    @torch.no_grad()
    def step(self, closure: Callable[[], Any] | None = None) -> Any:
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            for bucket in _by_shape(group["params"]):
                self._step_shape(bucket, group)
        return loss

    def _step_shape(self, params: list[Tensor], group: dict[str, Any]) -> None:
        shape = params[0].shape
        if len(shape) < 2:
            raise ValueError(f"NorMuon requires ndim >= 2; got shape {tuple(shape)}.")
        st = self.state[params[0]]
        tall = shape[-2] >= shape[-1]
        if "momentum_buffer" not in st:
            st["momentum_buffer"] = torch.zeros(len(params), *shape, dtype=params[0].dtype, device=params[0].device)
            st["second_moment"] = torch.zeros(
                (len(params), shape[-2], 1) if tall else (len(params), 1, shape[-1]),
                dtype=params[0].dtype,
                device=params[0].device,
            )
        grads = torch.stack([p.grad for p in params])  # type: ignore[misc]
        stacked = torch.stack(list(params))
        _normuon_update(
            grads, stacked, st["momentum_buffer"], st["second_moment"],
            momentum=group["momentum"], lr=group["lr"] * max(1.0, shape[-2] / shape[-1]) ** 0.5,
            weight_decay=group["weight_decay"], beta2=group["beta2"], ns_steps=group["ns_steps"],
            reduce_dim=-1 if tall else -2, coefficients=group["coefficients"],
        )  # fmt: skip
        torch._foreach_copy_(list(params), list(stacked.unbind(0)))  # noqa: SLF001
