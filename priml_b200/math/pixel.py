"""Pixel / video helpers (``priml/math/pixel.py:37-510``)."""

from __future__ import annotations

import io
import math
from collections.abc import Iterable, Sequence
from typing import Literal, NamedTuple

import numpy as np
import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200.math.basic import ceil_div
from priml_b200.math.custom_types import Tensorable, convert_to_tensor

__all__ = [
    "ImageShape",
    "ShapeBundle",
    "VideoShape",
    "compute_video_shapes",
    "decode_image_pil",
    "decode_jpeg_turbojpeg",
    "decode_webp_libwebp",
    "float2rgb",
    "interpolate",
    "patchify",
    "reconstruction_diffs",
    "rgb2float",
    "unpatchify",
]


def rgb2float(x: Tensorable) -> Tensor:
    """[0, 255] -> [-1, 1]."""
    return convert_to_tensor(x, dtype=torch.float32) / 127.5 - 1.0


def float2rgb(x: Tensorable) -> Tensor:
    """[-1, 1] -> uint8 [0, 255] (clamped, truncating)."""
    return (convert_to_tensor(x, dtype=torch.float32) * 127.5 + 127.5).clamp(0.0, 255.0).to(torch.uint8)


class ImageShape(NamedTuple):
    height: int
    width: int


class VideoShape(NamedTuple):
    frames: int
    height: int
    width: int


class ShapeBundle(NamedTuple):
    latent: VideoShape
    pixel_train: VideoShape
    pixel_full: VideoShape


def compute_video_shapes(nominal_resolution: int = 1080, aspect: float = 16 / 9, duration_sec: float = 5.0,
                         fps: float = 30.0,
                         compression: tuple[int, int, int] = VideoShape(frames=8, height=16, width=16)
                         ) -> ShapeBundle:  # fmt: skip
    """Latent and pixel shapes for a nominal resolution ("1080p") and aspect ratio.

    The frame area is ``(4/3 * nominal)^2`` split by the aspect ratio; the latent
    shape is the pixel shape divided by ``compression`` rounded up, and the
    training pixel shape is the latent shape times ``compression``. A zero
    duration means a single image.
    """
    side = nominal_resolution * 4.0 / 3.0
    r = math.sqrt(aspect)
    height, width = round(side / r), round(side * r)
    frames = 1 if duration_sec == 0 else round(duration_sec * fps)
    cf, ch, cw = compression
    latent = VideoShape(ceil_div(frames, cf), ceil_div(height, ch), ceil_div(width, cw))
    train = VideoShape(latent.frames * cf, latent.height * ch, latent.width * cw)
    full = VideoShape(1 if duration_sec == 0 else train.frames, height, width)
    for name, shape in (("latent", latent), ("training pixel", train), ("inference pixel", full)):
        if min(shape) <= 0:
            raise ValueError(f"invalid {name} shape {shape}")
    return ShapeBundle(latent, train, full)


def reconstruction_diffs(x: Tensor, y: Tensor, amplification: float = 3) -> Tensor:
    """``clamp(amplification * |x - y|, 0, 255)`` as uint8, for visual diffs."""
    x, y = convert_to_tensor(x, y, dtype=torch.float32)
    return (amplification * (x - y).abs()).clamp(0, 255).to(torch.uint8)


def patchify(x: Tensorable, patch_size: Iterable[int]) -> Tensor:
    """``... c (s1 p1) .. (sn pn) -> ... (c p1 .. pn) s1 .. sn``."""
    x = convert_to_tensor(x)
    ps = tuple(patch_size)
    n = len(ps)
    if x.ndim < n + 1:
        raise ValueError(f"{tuple(x.shape)} needs at least {n + 1} dimensions")
    lead = x.shape[: -n - 1]
    c = x.shape[-n - 1]
    split = [v for s, p in zip(x.shape[-n:], ps, strict=True) for v in (s // p, p)]
    y = x.reshape(*lead, c, *split)
    b = len(lead)
    # [..., c, s1, p1, ..., sn, pn] -> [..., c, p1..pn, s1..sn]
    order = list(range(b + 1)) + [b + 2 + 2 * i for i in range(n)] + [b + 1 + 2 * i for i in range(n)]
    y = y.permute(order)
    return y.reshape(*lead, c * math.prod(ps), *y.shape[-n:])


def unpatchify(x: Tensorable, patch_size: Iterable[int]) -> Tensor:
    """Inverse of :func:`patchify`."""
    x = convert_to_tensor(x)
    ps = tuple(patch_size)
    n = len(ps)
    lead = x.shape[: -n - 1]
    cp = x.shape[-n - 1]
    grid = x.shape[-n:]
    y = x.reshape(*lead, cp // math.prod(ps), *ps, *grid)
    b = len(lead) + 1
    order = list(range(b)) + [v for i in range(n) for v in (b + n + i, b + i)]
    y = y.permute(order)
    return y.reshape(*lead, cp // math.prod(ps), *[g * p for g, p in zip(grid, ps, strict=True)])


InterpolateMode = Literal["area", "area-variance-preserving", "bicubic", "bilinear", "linear", "nearest",
                          "nearest-exact", "trilinear", "cubic"]  # fmt: skip


def interpolate(input_: Tensorable, mode: InterpolateMode = "nearest", *, size: int | Sequence[int] = (),
                scale_factor: float | Sequence[int | float] = (), align_corners: bool = False,
                recompute_scale_factor: bool = False, antialias: bool = False, rank: int | None = None,
                channels_last: bool = False) -> Tensor:  # fmt: skip
    """``F.interpolate`` with the spatial rank inferred (from the mode prefix, ``size``,
    ``scale_factor`` or ``rank``), "linear"/"cubic" mapped to the rank's mode, any number
    of leading batch dims, channels-last input, and an ``area-variance-preserving``
    mode (adaptive sum-pool / sqrt(window))."""
    x = convert_to_tensor(input_)
    if mode.startswith("bi"):
        out_rank = 2
    elif mode.startswith("tri"):
        out_rank = 3
    elif isinstance(size, Sequence) and len(size) > 0:
        out_rank = len(size)
    elif isinstance(scale_factor, Sequence) and len(scale_factor) > 0:
        out_rank = len(scale_factor)
    elif rank is not None:
        out_rank = rank
    elif mode == "linear":
        out_rank = 1
    else:
        raise ValueError("cannot infer the spatial rank; pass size, scale_factor or rank")
    mode_map = {2: {"linear": "bilinear", "cubic": "bicubic"}, 3: {"linear": "trilinear"}}
    tmode = mode_map.get(out_rank, {}).get(mode, mode)
    size_t = (tuple(int(s) for s in size) if isinstance(size, Sequence) else (int(size),) * out_rank) or None
    sf_t = (tuple(float(s) for s in scale_factor) if isinstance(scale_factor, Sequence)
            else (float(scale_factor),) * out_rank) or None  # fmt: skip
    if x.ndim < out_rank:
        raise ValueError(f"a rank-{out_rank} interpolation needs at least {out_rank} dims, got {x.ndim}")
    if channels_last and x.ndim > out_rank:
        x = torch.movedim(x, -1, -out_rank - 1)
    squeeze = x.ndim == out_rank
    if squeeze:
        x = x[None]
    lead = x.shape[: -out_rank - 1]
    y = x.reshape(-1, *x.shape[-out_rank - 1 :])
    if tmode == "area-variance-preserving":
        from priml_b200.math.pooling import adaptive_avg_pool2d, adaptive_avg_pool3d

        if out_rank not in (2, 3):
            raise NotImplementedError("area-variance-preserving supports 2-D and 3-D only")
        target = size_t or tuple(int(s * f) for s, f in zip(y.shape[-out_rank:], sf_t or (), strict=True))
        y = (adaptive_avg_pool2d if out_rank == 2 else adaptive_avg_pool3d)(y, target, variance_preserving=True)
    else:
        linear_like = tmode.endswith("linear") or tmode.endswith("cubic")
        y = F.interpolate(y, size=size_t, scale_factor=None if size_t else sf_t, mode=tmode,
                          align_corners=align_corners if linear_like else None,
                          recompute_scale_factor=recompute_scale_factor if not size_t else None,
                          antialias=antialias)  # fmt: skip
    y = y.reshape(*lead, *y.shape[1:])
    if squeeze:
        y = y[0]
    if channels_last and y.ndim > out_rank:
        y = torch.movedim(y, -out_rank - 1, -1)
    return y


def _to_tensor(arr: np.ndarray | None, channels_first: bool) -> Tensor | None:
    if arr is None:
        return None
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if t.ndim == 2:
        t = t[..., None]
    return t.permute(2, 0, 1) if channels_first else t


def decode_image_pil(data: bytes, *, channels_first: bool = True, mode: str = "RGB") -> Tensor | None:
    """Decode an encoded image (any format PIL reads) to uint8 ``[C, H, W]``; None if unreadable."""
    try:
        from PIL import Image

        with Image.open(io.BytesIO(data)) as im:
            return _to_tensor(np.asarray(im.convert(mode)), channels_first)
    except Exception:  # noqa: BLE001 -- corrupt or unsupported input
        return None


def decode_jpeg_turbojpeg(data: bytes, *, channels_first: bool = True) -> Tensor | None:
    """JPEG through libjpeg-turbo when its Python binding is installed, else through PIL."""
    try:
        from turbojpeg import TurboJPEG  # type: ignore[import-not-found]
    except ImportError:
        return decode_image_pil(data, channels_first=channels_first)
    try:
        return _to_tensor(TurboJPEG().decode(data)[..., ::-1], channels_first)
    except Exception:  # noqa: BLE001
        return None


def decode_webp_libwebp(data: bytes, *, channels_first: bool = True) -> Tensor | None:
    """WebP through libwebp's binding when installed, else through PIL."""
    try:
        import webp  # type: ignore[import-not-found]
    except ImportError:
        return decode_image_pil(data, channels_first=channels_first)
    try:
        return _to_tensor(np.asarray(webp.WebPData.from_buffer(data).decode()), channels_first)
    except Exception:  # noqa: BLE001
        return None
