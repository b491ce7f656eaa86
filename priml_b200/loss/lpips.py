"""LPIPS perceptual distance and a per-video LPIPS loss (``priml/loss/lpips_loss.py:23-80``).

The reference wraps the third-party ``lpips`` package. This module implements
the metric itself (Zhang et al. 2018, "The Unreasonable Effectiveness of Deep
Features as a Perceptual Metric", arXiv:1801.03924):

1. inputs in ``[-1, 1]`` are shifted and scaled per channel to the statistics the
   backbone was trained on;
2. a convolutional backbone (torchvision VGG-16, AlexNet or SqueezeNet 1.1) gives
   feature maps at fixed taps;
3. each tap's features are unit-normalised over channels, the two images'
   difference is squared, weighted per channel by a non-negative 1x1 "lin" layer,
   averaged over space, and the taps are summed.

No weights are downloaded. The backbone starts from torchvision's random init
and the lin layers from ones (the unweighted "baseline" LPIPS); trained weights
load with ``load_state_dict`` -- :func:`remap_lpips_checkpoint` maps the lin
weights of an ``lpips`` package checkpoint (``lin{i}.model.1.weight``) to this
module's names (``lins.{i}.weight``), and ``backbone_weights`` loads a torchvision
state dict. The shift/scale constants are the published ones, kept alike so that
published lin weights mean the same thing here.
"""

from __future__ import annotations

import re
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.config import Fig

__all__ = ["LPIPS", "LPIPSLoss", "remap_lpips_checkpoint"]

# backbone name -> (torchvision constructor, index of each tap in `.features`, channels per tap)
_BACKBONES: dict[str, tuple[str, tuple[int, ...], tuple[int, ...]]] = {
    "vgg": ("vgg16", (3, 8, 15, 22, 29), (64, 128, 256, 512, 512)),
    "alex": ("alexnet", (1, 4, 7, 9, 11), (64, 192, 384, 256, 256)),
    "squeeze": ("squeezenet1_1", (1, 4, 7, 9, 10, 11, 12), (64, 128, 256, 384, 384, 512, 512)),
}
_SHIFT = (-0.030, -0.088, -0.188)  # published LPIPS input statistics for inputs in [-1, 1]
_SCALE = (0.458, 0.448, 0.450)


class LPIPS(nn.Module):
    """``forward(a, b)`` -> ``[N, 1, 1, 1]`` perceptual distances of ``[N, 3, H, W]`` images in ``[-1, 1]``."""

    def __init__(self, net: str = "vgg", backbone_weights: str | None = None) -> None:
        super().__init__()
        if net not in _BACKBONES:
            raise ValueError(f"net must be one of {sorted(_BACKBONES)}; got {net!r}.")
        import torchvision

        ctor, taps, channels = _BACKBONES[net]
        backbone = getattr(torchvision.models, ctor)(weights=None)
        if backbone_weights is not None:
            backbone.load_state_dict(torch.load(backbone_weights, map_location="cpu", weights_only=True))
        self.features = backbone.features[: taps[-1] + 1].requires_grad_(False)
        self.taps = taps
        self.lins = nn.ModuleList(nn.Conv2d(c, 1, 1, bias=False) for c in channels)
        for lin in self.lins:
            nn.init.ones_(lin.weight)
        self.lins.requires_grad_(False)
        self.register_buffer("shift", torch.tensor(_SHIFT).view(1, 3, 1, 1), persistent=False)
        self.register_buffer("scale", torch.tensor(_SCALE).view(1, 3, 1, 1), persistent=False)
        self.eval()

    def _taps(self, x: Tensor) -> list[Tensor]:
        out, want = [], set(self.taps)
        for i, layer in enumerate(self.features):
            x = layer(x)
            if i in want:
                out.append(x)
        return out

    def forward(self, a: Tensor, b: Tensor) -> Tensor:
        n = a.shape[0]
        both = torch.cat([a, b]).to(self.shift.dtype)
        feats = self._taps((both - self.shift) / self.scale)
        total = torch.zeros(n, 1, 1, 1, device=a.device, dtype=torch.float32)
        for f, lin in zip(feats, self.lins, strict=True):
            f = f.float()
            f = f / (f.square().sum(dim=1, keepdim=True).sqrt() + 1e-10)
            d = (f[:n] - f[n:]).square()
            total = total + lin(d.to(lin.weight.dtype)).float().mean(dim=(2, 3), keepdim=True)
        return total


def remap_lpips_checkpoint(state_dict: dict[str, Tensor]) -> dict[str, Tensor]:
    """``lpips`` package lin weights (``lin{i}.model.1.weight``) -> :class:`LPIPS` names (``lins.{i}.weight``)."""
    out = {}
    for k, v in state_dict.items():
        m = re.fullmatch(r"lin(\d+)\.model\.1\.weight", k)
        if m:
            out[f"lins.{m.group(1)}.weight"] = v
    return out


class LPIPSLoss(nn.Module):
    """Per-video LPIPS over a random subset of frames: ``{"loss": [B]}``.

    ``x`` and ``xhat`` are ``[B, C, T, H, W]``; up to ``max_num_random_frames``
    distinct frames (the same ones for every video) are compared, and each
    video's loss is the mean over them.
    """

    class Config(Fig["LPIPSLoss"]):
        max_num_random_frames: int = 2
        """Frames sampled per video (at most the number it has)."""
        net: str = "vgg"
        """Backbone: ``"vgg"``, ``"alex"`` or ``"squeeze"``."""
        weights: str | None = None
        """Optional state dict of :class:`LPIPS` (backbone and lin layers)."""

    def __init__(self, config: Config, criterion: nn.Module | None = None) -> None:
        super().__init__()
        self.max_num_random_frames = config.max_num_random_frames
        if criterion is None:
            criterion = LPIPS(config.net)
            if config.weights is not None:
                criterion.load_state_dict(torch.load(config.weights, map_location="cpu", weights_only=True),
                                          strict=False)  # fmt: skip
        self.lpips_criterion = criterion

    def forward(self, model_output: Any, *, x: Tensor, xhat: Tensor, **batch: Any) -> dict[str, Tensor]:
        del model_output, batch
        if x.ndim != 5:
            raise ValueError(f"expected [B, C, T, H, W] videos; got shape {tuple(x.shape)}.")
        t = x.shape[2]
        pick = torch.randperm(t, device=x.device)[: min(self.max_num_random_frames, t)]
        b, n = x.shape[0], pick.numel()

        def frames(v: Tensor) -> Tensor:
            return v.index_select(2, pick).transpose(1, 2).flatten(0, 1)  # [B * n, C, H, W]

        dist = self.lpips_criterion(frames(x), frames(xhat))
        return {"loss": dist.reshape(b, n).mean(dim=1)}
