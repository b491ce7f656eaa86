"""Diffusion training loss (``priml/loss/diffusion.py:23-140``).

One call draws a noise level per sample, corrupts the clean input, asks the
denoiser for its prediction and returns the per-sample squared error against
the configured target. The noise level is ``log t`` with ``t ~ U(0, 1)``,
optionally transformed, mapped to a log signal-to-noise ratio and from there to
the noise coefficient; the schedules and targets are the math library's
(:mod:`priml_b200.math.diffusion`). ``snr_gamma > 0`` applies Min-SNR-gamma
weighting (Hang et al. 2023, arXiv:2303.09556): each sample's loss is scaled by
``min(SNR, gamma) / SNR``.
"""

from __future__ import annotations

import math
from collections.abc import Callable
from typing import TypedDict

import torch
from torch import Tensor, nn

from priml_b200.config import Fig
from priml_b200.math.diffusion import (
    compute_log_alpha,
    log_sigma_from_log_snr_per_rectified_flow,
    log_snr_from_log_time_per_truncnormicdf,
    target_rectified_flow,
)
from priml_b200.math.numeric import safe_log

__all__ = ["DiffusionLoss"]


class DiffusionLoss(nn.Module):
    """``loss(denoiser, x0)`` with ``denoiser(x_noisy, sigma) -> model output``; rectified flow by default."""

    class Config(Fig["DiffusionLoss"]):
        logsnr_fn: Callable[[Tensor], Tensor] = log_snr_from_log_time_per_truncnormicdf
        """``log t -> log SNR``."""
        target_fn: Callable[..., tuple] = target_rectified_flow
        """Model output -> (target, prediction, x estimate, noise estimate)."""
        corruption_fn: Callable[[Tensor], Tensor] = log_sigma_from_log_snr_per_rectified_flow
        """``log SNR -> log sigma`` (the noise coefficient)."""
        time_transform: Callable[[Tensor], Tensor] | None = None
        """Optional map applied to ``log t`` first."""
        snr_gamma: float = 0.0
        """Min-SNR-gamma weight cap; 0 disables the weighting."""

    class Output(TypedDict):
        loss: Tensor  # [B]
        x_denoised: Tensor
        eps_denoised: Tensor
        log_snr: Tensor  # [B, 1, ...]
        log_sigma: Tensor

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.logsnr_fn = config.logsnr_fn
        self.target_fn = config.target_fn
        self.corruption_fn = config.corruption_fn
        self.time_transform = config.time_transform
        self.snr_gamma = config.snr_gamma

    def forward(self, denoiser: Callable[[Tensor, Tensor], Tensor], x0: Tensor) -> Output:
        per_sample = (x0.shape[0],) + (1,) * (x0.ndim - 1)
        log_t = safe_log(torch.rand(per_sample, device=x0.device, dtype=x0.dtype))
        if self.time_transform is not None:
            log_t = self.time_transform(log_t)
        noise = torch.randn_like(x0)
        log_snr = self.logsnr_fn(log_t)
        log_sigma = self.corruption_fn(log_snr)
        x_noisy = compute_log_alpha(log_snr, log_sigma).exp() * x0 + log_sigma.exp() * noise
        target, prediction, x_hat, eps_hat = self.target_fn(
            denoiser(x_noisy, log_sigma.exp()), x_noisy, log_snr, log_sigma, x_original=x0, eps_original=noise
        )
        loss = (target - prediction).square().flatten(1).mean(dim=1)
        if self.snr_gamma > 0:
            # min(SNR, gamma) / SNR in log space
            flat = log_snr.reshape(loss.shape[0])
            loss = loss * (flat.clamp(max=math.log(self.snr_gamma)) - flat).exp()
        return DiffusionLoss.Output(loss=loss, x_denoised=x_hat, eps_denoised=eps_hat, log_snr=log_snr,
                                    log_sigma=log_sigma)  # fmt: skip
