"""Ancestral DDPM / DDIM sampling (``priml/math/diffusion/sampling.py:37-500``).

One step from log-SNR ``l0`` (noisier) to ``l1`` (cleaner) given the model's
(x_clean, eps_clean): the DDPM posterior standard deviation is
``sigma_ddpm = sigma_1 sqrt(1 - snr_1^-1 snr_0)`` -- in log space
``log sigma_1 + log1mexp(l0 - l1) / 2`` -- and Song et al. 2020's eta scales the
random part, ``sigma_r = eta sigma_ddpm``, leaving the deterministic noise
coefficient ``sigma_d = sqrt(sigma_1^2 - sigma_r^2)``:
``mean = alpha_1 x_clean + sigma_d eps_clean``, ``std = sigma_r``.
eta = 0 is DDIM (deterministic), eta = 1 is DDPM.
"""

from __future__ import annotations

import functools
import math
from collections import deque
from collections.abc import Callable, Iterable, Iterator, Sequence
from typing import NamedTuple, Protocol

import torch
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor
from priml_b200.math.diffusion.schedule import compute_log_alpha, log_sigma_from_log_snr_per_rectified_flow
from priml_b200.math.diffusion.target import TargetFn, target_rectified_flow
from priml_b200.math.numeric import log1mexp

__all__ = ["SampleModelFn", "SampleOneStepFn", "SampleOneStepResult", "SampleResult", "ddim", "ddpm", "ddpm_ddim",
           "ddpm_ddim_step", "rescale_classifier_free_guidance", "sample", "sample_iter"]  # fmt: skip


class SampleOneStepResult(NamedTuple):
    x_clean: Tensor
    mean: Tensor
    log_std: Tensor


class SampleResult(NamedTuple):
    x_curr: Tensor
    x_clean: Tensor
    mean: Tensor
    log_std: Tensor
    model: Tensor


class SampleOneStepFn(Protocol):
    def __call__(self, model: Tensor, x_curr: Tensor, log_snr_curr: Tensor, log_snr_next: Tensor
                 ) -> SampleOneStepResult: ...  # fmt: skip


class SampleModelFn(Protocol):
    def __call__(self, x: Tensor, log_snr: Tensor, it: Tensor, num_steps: int, log_snr_next: Tensor) -> Tensor: ...


def ddpm_ddim_step(x_clean: Tensor, eps_clean: Tensor, log_snr_curr: Tensor, log_snr_next: Tensor,
                   log_sigma_next: Tensor, *, eta: float = 1) -> tuple[Tensor, Tensor]:  # fmt: skip
    """(mean, log std) of the step; requires ``log_snr_next > log_snr_curr``."""
    log_eta = math.log(eta) if eta > 0 else -math.inf
    log_sigma_r = log_sigma_next + 0.5 * log1mexp(log_snr_curr - log_snr_next) + log_eta
    log_sigma_d = log_sigma_next + 0.5 * log1mexp(2.0 * (log_sigma_r - log_sigma_next))
    alpha = torch.exp(compute_log_alpha(log_snr_next, log_sigma_next))
    return alpha * x_clean + torch.exp(log_sigma_d) * eps_clean, log_sigma_r


def ddpm_ddim(model: Tensor, x_curr: Tensorable, log_snr_curr: Tensorable, log_snr_next: Tensorable, *,
              corruption_fn: Callable[[Tensor], Tensor] = log_sigma_from_log_snr_per_rectified_flow,
              target_fn: TargetFn = target_rectified_flow, eta: float = 1) -> SampleOneStepResult:  # fmt: skip
    """Decompose the raw model output with ``target_fn`` and take one step."""
    x_curr, l0, l1 = convert_to_tensor(x_curr, log_snr_curr, log_snr_next)
    decomposed = target_fn(model, x_curr, l0, corruption_fn(l0))
    mean, log_std = ddpm_ddim_step(decomposed.x_clean, decomposed.eps_clean, l0, l1, corruption_fn(l1), eta=eta)
    return SampleOneStepResult(decomposed.x_clean, mean, log_std)


ddpm = functools.partial(ddpm_ddim, eta=1)
ddim = functools.partial(ddpm_ddim, eta=0)


def sample_iter(log_snr: Tensorable, model_fn: SampleModelFn, x_init: Tensorable,
                onestep_fn: Callable[..., SampleOneStepResult] = ddpm, *,
                noise_last_step: bool = False) -> Iterator[SampleResult]:  # fmt: skip
    """Yield every step of a run over ``log_snr[0] -> log_snr[-1]`` (``len - 1`` steps).
    Sampling noise is added after every step except (by default) the last, whose
    posterior mean is returned (Ho et al. 2020)."""
    x_curr, log_snr = convert_to_tensor(x_init, log_snr)
    steps = log_snr.shape[0] - 1
    if steps < 1:
        raise ValueError(f"log_snr needs at least 2 entries, got {steps + 1}")
    for i in range(steps):
        it = torch.tensor(i, dtype=torch.int64, device=x_curr.device)
        out = model_fn(x_curr, log_snr[i], it, steps, log_snr[i + 1])
        x_clean, mean, log_std = onestep_fn(out, x_curr, log_snr[i], log_snr[i + 1])
        last = i == steps - 1
        x_curr = mean if (last and not noise_last_step) else mean + torch.exp(log_std) * torch.randn_like(mean)
        yield SampleResult(x_curr, x_clean, mean, log_std, out)


def sample(log_snr: Tensorable, model_fn: SampleModelFn, x_init: Tensorable,
           onestep_fn: Callable[..., SampleOneStepResult] = ddpm, *, noise_last_step: bool = False,
           wrap_steps: Callable[[Iterable[SampleResult]], Iterable[SampleResult]] = lambda it: it) -> SampleResult:  # fmt: skip
    """Run :func:`sample_iter` to completion (through ``wrap_steps``) and return the last step."""
    last = deque(wrap_steps(sample_iter(log_snr, model_fn, x_init, onestep_fn, noise_last_step=noise_last_step)),
                 maxlen=1)  # fmt: skip
    if not last:
        raise ValueError("sampling produced no steps")
    return last[0]


def rescale_classifier_free_guidance(guided: Tensor, unguided: Tensor, *, strength: float = 0.0, eps: float = 1e-9,
                                     spatial_dims: Sequence[int] | None = None) -> Tensor:  # fmt: skip
    """Blend ``guided`` with its rescaling to ``unguided``'s standard deviation (Lin et al. 2024, eq. 6)."""
    dims = tuple(spatial_dims) if spatial_dims is not None else tuple(range(1, guided.ndim))
    rescaled = guided * (unguided.std(dim=dims, keepdim=True) / (guided.std(dim=dims, keepdim=True) + eps))
    return torch.lerp(guided, rescaled, strength)
