"""Rotary position embeddings (``priml/model/rope.py:23-666``).

``RoPE(positions)`` returns half-dim ``(cos, sin)`` of shape ``[..., S, 1, D/2]``
(fp32 unless ``dtype`` is set); ``RoPE.rotate`` applies the half-split (HF) or
interleaved rotation in fp32 and rounds once. On CUDA the half-split case is one
fused kernel (``priml_b200.ops.rotary``) reading q, k and the table once.

Inverse frequencies are rebuilt on every device move: ``base ** x`` differs in
the last bit between host and device math libraries, so a device-built table is
the one a device run must use.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterable, Sequence
from dataclasses import KW_ONLY, dataclass
from typing import Any, Literal

import torch
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig, Makes
from priml_b200.math.basic import broadcast_sequences

__all__ = ["RoPE", "RoPEMixed", "YarnScaling", "rotate_conjugate"]


@dataclass(frozen=True, slots=True, kw_only=True)
class YarnScaling:
    """YaRN (Peng et al. 2023, arXiv:2309.00071) in the DeepSeek-V3 convention."""

    factor: float
    original_max_position_embeddings: int
    beta_fast: float = 32.0
    beta_slow: float = 1.0
    mscale: float = 1.0
    mscale_all_dim: float = 0.0


class RoPE(nn.Module):
    """N-axis rotary embedding with fixed frequencies."""

    class Config(Fig["RoPE"], kw_only=False):
        channels_head: int | Iterable[int] = 64
        """Rotated channels per axis (a scalar is split across axes in cat mode)."""
        _: KW_ONLY
        base: float | Iterable[float] = 10e3
        reduction_mode: Literal["cat", "sum"] = "cat"
        yarn: YarnScaling | None = None
        hf_inv_freq: bool = False
        """Use ``1 / base ** (arange(0, c, 2) / c)`` (HF) instead of the fp64
        ``exp(linspace(0, log(base) * (2/c - 1), c/2))``."""
        dtype: torch.dtype | None = None
        """Width of the returned factors (None = fp32)."""

    def __init__(self, config: Config) -> None:
        super().__init__()
        c: Any = config.channels_head
        base: Any = config.base
        self.reduction_mode = config.reduction_mode
        if self.reduction_mode == "cat" and isinstance(c, int) and isinstance(base, Sequence) and len(base) > 1:
            c = self._split_dim(c, len(base))
        cs, bs = broadcast_sequences(c, base)
        self.channels_head = tuple(int(d) for d in cs)
        self.base = tuple(float(b) for b in bs)
        self._hf_inv_freq = config.hf_inv_freq
        self._yarn = config.yarn
        self._mscale = 1.0
        self._inv_freqs: list[Tensor] = []
        self._build_inv_freqs(torch.device("cpu"))
        if all(not f.numel() for f in self._inv_freqs):
            raise ValueError(f"At least one dim must be nonzero, got {self.channels_head}.")
        self._dtype = nn.Buffer(torch.empty(0, dtype=config.dtype), persistent=False)
        self._table_cache: dict[Any, tuple[Tensor, Tensor]] = {}

    @property
    def dtype(self) -> torch.dtype:
        return self._dtype.dtype

    @property
    def device(self) -> torch.device:
        return self._dtype.device

    def forward(self, positions: Tensor) -> tuple[Tensor, Tensor]:
        if positions.ndim == 1:
            positions = positions.unsqueeze(-1)
        pos = positions.to(dtype=torch.float32).split(1, dim=-1)
        parts = [
            p.unsqueeze(-1) * f.to(dtype=torch.float32, device=p.device)
            for p, f in zip(pos, self._inv_freqs, strict=True)
            if f.numel()
        ]
        if self.reduction_mode == "cat":
            emb = torch.cat(parts, dim=-1)
        elif self.reduction_mode == "sum":
            emb = sum(parts[1:], parts[0])
        else:
            raise ValueError(f"Unknown reduction_mode {self.reduction_mode!r}.")
        cos = emb.cos() * self._mscale
        sin = emb.sin() * self._mscale
        return cos.to(dtype=self.dtype, device=self.device), sin.to(dtype=self.dtype, device=self.device)

    def table(self, seq_len: int, device: torch.device) -> tuple[Tensor, Tensor]:
        """Cached ``(cos, sin)`` for positions ``0..seq_len-1`` (``[S, 1, D/2]``)."""
        key = (seq_len, str(device))
        hit = self._table_cache.get(key)
        if hit is None:
            hit = self(torch.arange(seq_len, device=device))
            self._table_cache = {key: hit}
        return hit

    @classmethod
    def rotate(cls, q: Tensor, k: Tensor, cos: Tensor, sin: Tensor, interleave: bool = False) -> tuple[Tensor, Tensor]:
        """Rotate ``[..., S, H, D]`` q/k by half-dim factors ``[..., S', H|1, D_rot/2]``.

        ``S' < S`` pads with identity; ``D_rot < D`` rotates only the first
        ``D_rot`` channels.
        """
        seq_dim = -3
        s, s_rot = q.shape[seq_dim], cos.shape[seq_dim]
        if s_rot < s:
            pad = list(cos.shape)
            pad[seq_dim] = s - s_rot
            cos = torch.cat([cos, torch.ones(pad, dtype=cos.dtype, device=cos.device)], dim=seq_dim)
            sin = torch.cat([sin, torch.zeros(pad, dtype=sin.dtype, device=sin.device)], dim=seq_dim)
        rot = cos.shape[-1] * 2
        d = q.shape[-1]
        if not interleave and rot == d and q.ndim == 4 and cos.ndim == 3 and cos.shape[-2] == 1:
            return ops.rotary(q, k, cos, sin)
        if rot < d:
            qr, qp = q[..., :rot], q[..., rot:]
            kr, kp = k[..., :rot], k[..., rot:]
            return (
                torch.cat([cls._rotate(qr, cos, sin, interleave), qp], dim=-1),
                torch.cat([cls._rotate(kr, cos, sin, interleave), kp], dim=-1),
            )
        return cls._rotate(q, cos, sin, interleave), cls._rotate(k, cos, sin, interleave)

    @classmethod
    def _rotate(cls, x: Tensor, cos: Tensor, sin: Tensor, interleave: bool) -> Tensor:
        dtype = x.dtype
        x = x.float()
        if interleave:
            x0, x1 = x[..., 0::2], x[..., 1::2]
            out = torch.zeros_like(x)
            out[..., 0::2] = x0 * cos - x1 * sin
            out[..., 1::2] = x1 * cos + x0 * sin
        else:
            half = x.shape[-1] // 2
            x0, x1 = x[..., :half], x[..., half:]
            out = torch.cat([x0 * cos - x1 * sin, x1 * cos + x0 * sin], dim=-1)
        return out.to(dtype)

    @classmethod
    def smallest_recommended_base(
        cls, dim: int | Iterable[int], max_positions: int | Iterable[int]
    ) -> float | tuple[float, ...]:
        """Smallest base whose slowest wavelength covers ``max_positions``:
        ``((m - 1) / 2pi) ** (c / (c - 2))``."""
        dims, maxpos = broadcast_sequences(dim, max_positions)
        out: list[float] = []
        for c, m in zip(dims, maxpos, strict=True):
            if c == 0:
                out.append(0.0)
                continue
            cls._validate_c(c)
            out.append(((m - 1) / (2 * math.pi)) ** (c / (c - 2)))
        return out[0] if len(out) == 1 else tuple(out)

    def _apply(self, fn: Callable[..., Any], recurse: bool = True) -> RoPE:
        super()._apply(fn, recurse)
        self._build_inv_freqs(self._dtype.device)
        self._table_cache = {}
        return self

    def _build_inv_freqs(self, device: torch.device) -> None:
        def axis(base: float, width: int) -> Tensor:
            if width == 0:  # an axis without rotary channels
                return torch.empty(0, device=device)
            self._validate_c(width)
            freqs = self._make_inv_freqs(base, width, hf=self._hf_inv_freq, device=device)
            if self._yarn is not None:
                freqs, self._mscale = _yarn_apply(freqs, base, width, self._yarn)
            return freqs.unsqueeze(-2)

        self._inv_freqs = [axis(b, c) for b, c in zip(self.base, self.channels_head, strict=True)]

    @classmethod
    def _make_inv_freqs(cls, b: float, c: int, *, hf: bool = False, device: torch.device | None = None) -> Tensor:
        if hf:
            ch = torch.arange(0, c, 2, dtype=torch.int64, device=device).float()
            return 1.0 / (b ** (ch / c))
        return torch.linspace(0, math.log(b) * (-1 + 2 / c), c // 2, dtype=torch.float64, device=device).exp().float()

    @classmethod
    def _validate_c(cls, c: int) -> None:
        if c < 2 or c % 2:
            raise ValueError(f"a rotary axis needs an even number (at least 2) of channels; got {c}.")

    @classmethod
    def _split_dim(cls, total: int, naxes: int) -> list[int]:
        if total % 2 or total < 2 * naxes:
            raise ValueError(f"{total} rotary channels cannot be shared as channel pairs by {naxes} axes.")
        per = total // naxes // 2 * 2
        dims = [per] * naxes
        for i in range((total - per * naxes) // 2):
            dims[i] += 2
        return dims


def rotate_conjugate(x: Tensor, *, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotate channel pairs ``(i, i+D/2)`` by ``-theta`` at the input's own precision."""
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    return torch.cat([a * cos + b * sin, a * (-sin) + b * cos], dim=-1)


def _yarn_mscale(scale: float, mscale: float) -> float:
    return 1.0 if scale <= 1.0 else 0.1 * math.log(scale) * mscale + 1.0


def _yarn_correction_range(low_rot: float, high_rot: float, dim: int, base: float, max_pos: int) -> tuple[float, float]:
    def corr(n: float) -> float:
        return dim * math.log(max_pos / (n * 2 * math.pi)) / (2 * math.log(base))

    return max(math.floor(corr(low_rot)), 0), min(math.ceil(corr(high_rot)), dim - 1)


def _yarn_apply(inv_freq: Tensor, base: float, dim: int, yarn: YarnScaling) -> tuple[Tensor, float]:
    """Blend extrapolated (high-frequency) and ``/factor``-interpolated
    (low-frequency) inverse frequencies with a linear ramp over channel index."""
    lo, hi = _yarn_correction_range(yarn.beta_fast, yarn.beta_slow, dim, base, yarn.original_max_position_embeddings)
    lo_f, hi_f = float(lo), float(hi)
    if hi_f == lo_f:
        hi_f = lo_f + 1e-3
    ramp = ((torch.arange(dim // 2, dtype=torch.float32, device=inv_freq.device) - lo_f) / (hi_f - lo_f)).clamp(0.0, 1.0)
    keep = 1.0 - ramp
    blended = inv_freq * keep + (inv_freq / yarn.factor) * (1.0 - keep)
    if yarn.mscale_all_dim != 0:
        m = _yarn_mscale(yarn.factor, yarn.mscale) / _yarn_mscale(yarn.factor, yarn.mscale_all_dim)
    else:
        m = _yarn_mscale(yarn.factor, yarn.mscale)
    return blended, m


class RoPEMixed(RoPE):
    """RoPE with per-head frequencies scaled by random unit directions
    (RoPE-Mixed, Heo et al. 2024, arXiv:2403.13298); optionally learnable."""

    class Config(Makes["RoPEMixed"], RoPE.Config):
        heads: int = 1
        learnable: bool = False

    def __init__(self, config: Config) -> None:
        super().__init__(config)
        self.heads = config.heads
        self.learnable = config.learnable
        if config.reduction_mode == "sum":
            active = {f.shape[-1] for f in self._inv_freqs if f.numel()}
            if len(active) > 1:
                raise ValueError(f"Sum mode requires uniform dims, got {active}.")
        self._base_inv_freqs = [f.detach().clone() for f in self._inv_freqs]
        col = torch.empty(self.heads, 1) if self.heads > 1 else None
        self._inv_freqs = nn.ParameterList(  # type: ignore[assignment]
            nn.Parameter(torch.empty_like(f * col if col is not None else f), requires_grad=self.learnable)
            if f.numel()
            else nn.Parameter(torch.empty(0), requires_grad=False)
            for f in self._base_inv_freqs
        )
        self.reset_parameters()

    def reset_parameters(self) -> None:
        active = sum(1 for f in self._base_inv_freqs if f.numel())
        directions = None
        if self.heads > 1:
            directions = nn.functional.normalize(nn.init.trunc_normal_(torch.empty(active, self.heads, 1), std=1.0), dim=0)
        with torch.no_grad():
            j = 0
            for param, base in zip(self._inv_freqs, self._base_inv_freqs, strict=True):
                if base.numel():
                    param.copy_((base * directions[j] if directions is not None else base).to(param))
                    j += 1

    def _apply(self, fn: Callable[..., Any], recurse: bool = True) -> RoPEMixed:
        saved = [f.data.clone() for f in self._inv_freqs]
        nn.Module._apply(self, fn, recurse)
        for i, f in enumerate(saved):
            self._inv_freqs[i].data = f.to(device=self._dtype.device)
        self._table_cache = {}
        return self
