"""Convolution, diffusion-transformer and mixer blocks (``priml/model/conv.py``,
``mmdit.py``, ``mlpmixer.py``, ``patchify.py``, ``whitening.py``)."""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import KW_ONLY, dataclass, field
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable
from priml_b200.models.attention import MultiStreamAttention
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, propagate_attr
from priml_b200.models.init import InitFn, call_init, kaiming_uniform
from priml_b200.models.linear import Linear
from priml_b200.models.norm import LayerNorm, RMSNorm
from priml_b200.models.swiglu import SwiGLU

__all__ = ["AdaLNZero", "Conv1d", "Conv2d", "Conv3d", "MLPMixerBlock", "MMDiTBlock", "PCAWhiteningConv2d",
           "Patchify", "Unpatchify"]  # fmt: skip


def _conv_cls(base: type[nn.Module], name: str) -> type[nn.Module]:
    class _Conv(base):  # type: ignore[valid-type, misc]
        class Config(Fig[name], kw_only=False):
            channels_in: int = -1
            channels_out: int = -1
            _: KW_ONLY
            kernel_size: Any = 3
            stride: Any = 1
            padding: Any = "same"
            dilation: Any = 1
            groups: int = 1
            bias: bool = False
            depth: int = -1
            device: Any = None
            dtype: Any = None
            init_weight: InitFn = kaiming_uniform
            init_bias: InitFn = nn.init.zeros_

            def finalize(self):  # noqa: ANN201
                if self.channels_out == -1:
                    self.channels_out = self.channels_in
                return super().finalize()

        def __init__(self, config: Any) -> None:
            self._init_w, self._init_b, self.depth = config.init_weight, config.init_bias, config.depth
            super().__init__(config.channels_in, config.channels_out, config.kernel_size, stride=config.stride,
                             padding=config.padding, dilation=config.dilation, groups=config.groups, bias=config.bias,
                             device=config.device, dtype=config.dtype)  # fmt: skip

        def reset_parameters(self) -> None:
            if not hasattr(self, "_init_w"):
                return super().reset_parameters()
            call_init(self._init_w, self.weight, depth=self.depth)
            if self.bias is not None:
                call_init(self._init_b, self.bias, depth=self.depth)
            return None

    _Conv.__name__ = _Conv.__qualname__ = name
    _Conv.Config.__qualname__ = f"{name}.Config"
    return _Conv


Conv1d = _conv_cls(nn.Conv1d, "Conv1d")
Conv2d = _conv_cls(nn.Conv2d, "Conv2d")
Conv3d = _conv_cls(nn.Conv3d, "Conv3d")


class AdaLNZero(nn.Module):
    """Adaptive LayerNorm-zero modulation: ``cond -> (scale, shift, gate) x 2``,
    projection zero-initialized so a fresh block is the identity."""

    @dataclass
    class Output:
        attn_scale: Tensor
        attn_shift: Tensor
        attn_gate: Tensor
        ffn_scale: Tensor
        ffn_shift: Tensor
        ffn_gate: Tensor

    class Config(Fig["AdaLNZero"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        cond_dim: int = -1

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.proj = nn.Linear(config.cond_dim, 6 * config.channels_in)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.zeros_(self.proj.weight)
        nn.init.zeros_(self.proj.bias)

    def forward(self, c: Tensor) -> Output:
        parts = self.proj(F.silu(c)).unsqueeze(-2).chunk(6, dim=-1)
        return AdaLNZero.Output(*parts)


class MMDiTBlock(nn.Module):
    """N token streams with joint attention; each stream its own norms / FFN and
    optional AdaLN-zero conditioning (``priml/model/mmdit.py:111-293``). Submodule names
    (``norms1``, ``norms2``, ``ffns``, ``adalns``) give the reference's state-dict keys."""

    class Config(Fig["MMDiTBlock"], kw_only=False):
        channels_in: int = 768
        _: KW_ONLY
        num_streams: int = 2
        attn: Makeable[nn.Module] = field(default_factory=lambda: MultiStreamAttention.Config(heads=12))
        cond_dim: int = 0
        ffn: Makeable[nn.Module] = field(default_factory=SwiGLU.Config)
        depth: int = -1

        def finalize(self):  # noqa: ANN201
            propagate_attr(self.attn, "channels_in", self.channels_in)
            propagate_attr(self.attn, "num_streams", self.num_streams)
            propagate_attr(self.ffn, "channels_in", self.channels_in, protocol=ChannelsIn)
            propagate_attr(self.ffn, "channels_out", self.channels_in, protocol=ChannelsOut)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        c, n = config.channels_in, config.num_streams
        self.attn = config.attn.make()
        self.norms1 = nn.ModuleList(LayerNorm.Config(c).make() for _ in range(n))
        self.norms2 = nn.ModuleList(LayerNorm.Config(c).make() for _ in range(n))
        self.ffns = nn.ModuleList(config.ffn.make() for _ in range(n))
        self.adalns = (
            nn.ModuleList(AdaLNZero.Config(c, cond_dim=config.cond_dim).make() for _ in range(n))
            if config.cond_dim > 0
            else None
        )

    def forward(self, xs: Sequence[Tensor], c: Tensor | Sequence[Tensor] | None = None, **kwargs: Any) -> list[Tensor]:
        del kwargs
        n = len(xs)
        conds = [c] * n if isinstance(c, Tensor) or c is None else list(c)
        mods = [self.adalns[i](conds[i]) if self.adalns is not None and conds[i] is not None else None for i in range(n)]
        normed = []
        for i, x in enumerate(xs):
            h = self.norms1[i](x)
            if mods[i] is not None:
                h = h * (1 + mods[i].attn_scale) + mods[i].attn_shift
            normed.append(h)
        attn = self.attn(normed)
        out = []
        for i, x in enumerate(xs):
            a = attn[i] * mods[i].attn_gate if mods[i] is not None else attn[i]
            x = x + a
            h = self.norms2[i](x)
            if mods[i] is not None:
                h = h * (1 + mods[i].ffn_scale) + mods[i].ffn_shift
            f = self.ffns[i](h)
            out.append(x + (f * mods[i].ffn_gate if mods[i] is not None else f))
        return out


class MLPMixerBlock(nn.Module):
    """Token mixing across the sequence axis then channel mixing (Tolstikhin et al. 2021)."""

    class Config(Fig["MLPMixerBlock"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        seq_len: int = -1
        token_mixer: Makeable[nn.Module] = field(default_factory=SwiGLU.Config)
        channel_mixer: Makeable[nn.Module] = field(default_factory=SwiGLU.Config)
        norm_token: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        norm_channel: Makeable[nn.Module] = field(default_factory=RMSNorm.Config)
        prenorm: bool = True
        depth: int = -1

        def finalize(self):  # noqa: ANN201
            propagate_attr(self.token_mixer, "channels_in", self.seq_len, protocol=ChannelsIn)
            propagate_attr(self.token_mixer, "channels_out", self.seq_len, protocol=ChannelsOut)
            propagate_attr(self.channel_mixer, "channels_in", self.channels_in, protocol=ChannelsIn)
            propagate_attr(self.channel_mixer, "channels_out", self.channels_in, protocol=ChannelsOut)
            for n in (self.norm_token, self.norm_channel):
                propagate_attr(n, "channels_in", self.channels_in, protocol=ChannelsIn)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.prenorm = config.prenorm
        self.token_mixer = config.token_mixer.make()
        self.channel_mixer = config.channel_mixer.make()
        self.norm_token = config.norm_token.make()
        self.norm_channel = config.norm_channel.make()

    def reset_parameters(self) -> None:
        for m in (self.token_mixer, self.channel_mixer, self.norm_token, self.norm_channel):
            if hasattr(m, "reset_parameters"):
                m.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        if self.prenorm:
            x = x + self.token_mixer(self.norm_token(x).transpose(-1, -2)).transpose(-1, -2)
            return x + self.channel_mixer(self.norm_channel(x))
        x = self.norm_token(x + self.token_mixer(x.transpose(-1, -2)).transpose(-1, -2))
        return self.norm_channel(x + self.channel_mixer(x))


class Patchify(nn.Module):
    """``[B, C, *spatial]`` -> ``[B, N_patches, C * prod(patch)]`` (non-overlapping)."""

    class Config(Fig["Patchify"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        patch_size: list[int] = field(default_factory=lambda: [2, 2])

        @property
        def channels_out(self) -> int:
            n = 1
            for p in self.patch_size:
                n *= p
            return self.channels_in * n

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.patch = list(config.patch_size)

    def forward(self, x: Tensor) -> Tensor:
        b, c, *sp = x.shape
        nd = len(self.patch)
        grid = [s // p for s, p in zip(sp, self.patch, strict=True)]
        shape = [b, c] + [v for g, p in zip(grid, self.patch, strict=True) for v in (g, p)]
        x = x.reshape(shape)
        perm = [0] + [2 + 2 * i for i in range(nd)] + [1] + [3 + 2 * i for i in range(nd)]
        return x.permute(perm).reshape(b, -1, c * int(torch.tensor(self.patch).prod()))


class Unpatchify(nn.Module):
    """Inverse of :class:`Patchify` for a given spatial grid."""

    class Config(Fig["Unpatchify"], kw_only=False):
        channels_out: int = -1
        _: KW_ONLY
        patch_size: list[int] = field(default_factory=lambda: [2, 2])

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.patch = list(config.patch_size)
        self.channels = config.channels_out

    def forward(self, x: Tensor, grid: Sequence[int]) -> Tensor:
        b = x.shape[0]
        nd = len(self.patch)
        x = x.reshape([b, *grid, self.channels, *self.patch])
        perm = [0, nd + 1] + [v for i in range(nd) for v in (1 + i, nd + 2 + i)]
        return x.permute(perm).reshape([b, self.channels] + [g * p for g, p in zip(grid, self.patch, strict=True)])


class PCAWhiteningConv2d(nn.Conv2d):
    """Frozen patch-whitening convolution fit by PCA on training patches
    (Page 2019 / Keller Jordan's CIFAR-10 speedruns): filters = eigenvectors / sqrt(eigenvalues + eps)."""

    def __init__(self, channels_in: int, kernel_size: int = 2) -> None:
        super().__init__(channels_in, channels_in * kernel_size * kernel_size * 2, kernel_size, bias=False)
        self.weight.requires_grad_(False)

    @torch.no_grad()
    def fit(self, train_images: Tensor, eps: float = 5e-4) -> None:
        k = self.kernel_size[0]
        patches = train_images.unfold(2, k, 1).unfold(3, k, 1).transpose(1, 3).reshape(-1, self.in_channels * k * k)
        patches = patches.float() - patches.float().mean(0)
        cov = patches.T @ patches / patches.shape[0]
        evals, evecs = torch.linalg.eigh(cov)
        w = (evecs.T / torch.sqrt(evals + eps)[:, None]).flip(0).reshape(-1, self.in_channels, k, k)
        self.weight.copy_(torch.cat([w, -w], dim=0))
