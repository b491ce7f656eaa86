"""Batched image augmentation on device (``priml/data/augmentation_gpu.py:14-112``).

Random draws (crop offsets, flip flags, cutout corners) are made with torch on
the images' device; on CUDA the pad + crop + flip + cutout pipeline then runs as
one fused kernel (one read per output pixel, no padded copy), elsewhere as the
equivalent torch ops. ``pad_crop_flip(..., draws=...)`` replays given draws.
"""

from __future__ import annotations

from typing import NamedTuple

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200 import ops

__all__ = ["AugmentDraws", "cutout", "draw", "flip_lr", "pad_crop_flip", "random_crop"]


def flip_lr(images: Tensor) -> Tensor:
    """Horizontal flip of each image with probability 1/2."""
    mask = torch.rand(images.shape[0], device=images.device) < 0.5
    return torch.where(mask.view(-1, 1, 1, 1), images.flip(-1), images)


def _crop_at(images: Tensor, dy: Tensor, dx: Tensor, crop: int) -> Tensor:
    b, c, h, w = images.shape
    rows = dy.view(b, 1, 1, 1) + torch.arange(crop, device=images.device).view(1, 1, -1, 1)
    cols = dx.view(b, 1, 1, 1) + torch.arange(crop, device=images.device).view(1, 1, 1, -1)
    idx = (rows * w + cols).expand(b, c, crop, crop).reshape(b, c, -1)
    return images.reshape(b, c, -1).gather(2, idx).reshape(b, c, crop, crop)


def random_crop(images: Tensor, crop_size: int) -> Tensor:
    """Per-image uniform crop of a pre-padded square batch (offset in ``[0, 2 * ((H - crop) // 2)]``)."""
    b, _, h, w = images.shape
    if crop_size > h or crop_size > w:
        raise ValueError(f"crop_size={crop_size} exceeds the input ({h}x{w}); pad first")
    slack = 2 * ((h - crop_size) // 2)
    dy = torch.randint(0, slack + 1, (b,), device=images.device)
    dx = torch.randint(0, slack + 1, (b,), device=images.device)
    return _crop_at(images, dy, dx, crop_size)


def _cut_at(images: Tensor, cy: Tensor, cx: Tensor, size: int) -> Tensor:
    b, _, h, w = images.shape
    ys = torch.arange(h, device=images.device).view(1, 1, -1, 1)
    xs = torch.arange(w, device=images.device).view(1, 1, 1, -1)
    cy, cx = cy.view(b, 1, 1, 1), cx.view(b, 1, 1, 1)
    return images.masked_fill((ys >= cy) & (ys < cy + size) & (xs >= cx) & (xs < cx + size), 0)


def cutout(images: Tensor, size: int) -> Tensor:
    """Zero a ``size`` x ``size`` square whose corner is uniform over the image (clipped at edges)."""
    b, _, h, w = images.shape
    return _cut_at(images, torch.randint(0, h, (b,), device=images.device),
                   torch.randint(0, w, (b,), device=images.device), size)  # fmt: skip


class AugmentDraws(NamedTuple):
    dy: Tensor  # int32 [B]
    dx: Tensor
    flip: Tensor | None  # uint8 [B]
    cy: Tensor
    cx: Tensor


def draw(batch: int, crop_size: int, height: int, pad: int, flip: bool | None, device: torch.device) -> AugmentDraws:
    slack = 2 * ((height + 2 * pad - crop_size) // 2)
    dy = torch.randint(0, slack + 1, (batch,), device=device, dtype=torch.int32)
    dx = torch.randint(0, slack + 1, (batch,), device=device, dtype=torch.int32)
    if flip is None:
        fl = (torch.rand(batch, device=device) < 0.5).to(torch.uint8)
    elif flip:
        fl = torch.ones(batch, dtype=torch.uint8, device=device)
    else:
        fl = None
    cy = torch.randint(0, crop_size, (batch,), device=device, dtype=torch.int32)
    cx = torch.randint(0, crop_size, (batch,), device=device, dtype=torch.int32)
    return AugmentDraws(dy, dx, fl, cy, cx)


_MODES = {"constant": 0, "replicate": 1, "reflect": 2}


def pad_crop_flip(images: Tensor, crop_size: int, *, pad: int = 2, pad_mode: str = "reflect", flip: bool | None = None,
                  cutout_size: int = 0, draws: AugmentDraws | None = None) -> Tensor:  # fmt: skip
    """Pad by ``pad`` on every side, crop ``crop_size`` at a random offset, flip (random per
    image when ``flip`` is None), then cut out a square; contiguous ``[B, C, crop, crop]``."""
    b, _, h, _ = images.shape
    d = draws if draws is not None else draw(b, crop_size, h, pad, flip, images.device)
    if images.is_cuda and ops.use_native(images) and pad_mode in _MODES and images.is_contiguous():
        return ops.native().augment_pad_crop_flip_cutout(images, crop_size, pad, _MODES[pad_mode], 0.0, d.dy, d.dx,
                                                          d.flip, d.cy, d.cx, cutout_size)  # fmt: skip
    padded = F.pad(images, (pad,) * 4, mode=pad_mode) if pad > 0 else images
    out = _crop_at(padded, d.dy.long(), d.dx.long(), crop_size)
    if d.flip is not None:
        out = torch.where(d.flip.bool().view(-1, 1, 1, 1), out.flip(-1), out)
    if cutout_size > 0:
        out = _cut_at(out, d.cy.long(), d.cx.long(), cutout_size)
    return out.contiguous()
