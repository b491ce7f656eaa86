"""CIFAR-10 networks (``priml/baselines/cifar10/model.py:40-558``).

* ``ResNet``: pre-activation residual stages (norm, activation, conv), a
  stride-2 first block per later stage, global average pool, linear head.
* ``SpeedNet``: the speedrun design -- a frozen PCA patch-whitening conv fitted
  on training images, then wide ``ConvBlock`` stages (conv, max-pool, affine-free
  batch norm, activation; a residual over the last two convs), max-pool, and a
  head scaled by ``1 / channels``.

Convolutions run channels-last in bf16 under autocast through cuDNN (library
convolutions; the network's hot path is small 3x3 convs that cuDNN's sm_100
kernels already cover).
"""

from __future__ import annotations

from dataclasses import field
from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable, copy_tree
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, propagate_attr
from priml_b200.models.init import call_init
from priml_b200.models.vision import PCAWhiteningConv2d

__all__ = ["ConvBlock", "ResNet", "ResidualBlock", "ScaledLinear", "SpeedNet"]


def _activation(act: Any) -> Any:
    return act.make() if hasattr(act, "make") else act


def _block_grid(block: Any, num_stages: int, per_stage: int) -> list[list[Any]]:
    """Stage-grouped copies of a block template (or an explicit flat list)."""
    if isinstance(block, list):
        if len(block) != num_stages * per_stage:
            raise ValueError(f"block list must hold {num_stages * per_stage} configs; got {len(block)}.")
        flat = block
    else:
        flat = [copy_tree(block) for _ in range(num_stages * per_stage)]
    return [flat[i * per_stage : (i + 1) * per_stage] for i in range(num_stages)]


class ResidualBlock(nn.Module):
    class Config(Fig["ResidualBlock"]):
        channels_in: int = -1
        channels_out: int = -1
        stride: int = 1
        activation: Any = torch.relu
        norm_momentum: float = 0.1

        def finalize(self):  # noqa: ANN201
            if self.channels_in == -1:
                self.channels_in = self.channels_out
            if self.channels_out == -1:
                self.channels_out = self.channels_in
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        c_in, c_out = config.channels_in, config.channels_out
        self.norm1 = nn.BatchNorm2d(c_in, momentum=config.norm_momentum)
        self.conv1 = nn.Conv2d(c_in, c_out, 3, stride=config.stride, padding=1, bias=False)
        self.norm2 = nn.BatchNorm2d(c_out, momentum=config.norm_momentum)
        self.conv2 = nn.Conv2d(c_out, c_out, 3, padding=1, bias=False)
        self.act = _activation(config.activation)
        needs = config.stride != 1 or c_in != c_out
        self.shortcut = nn.Conv2d(c_in, c_out, 1, stride=config.stride, bias=False) if needs else nn.Identity()

    def forward(self, x: Tensor) -> Tensor:
        h = self.act(self.norm1(x))  # the shortcut reads the post-activation tensor
        return self.shortcut(h) + self.conv2(self.act(self.norm2(self.conv1(h))))


class ConvBlock(nn.Module):
    class Config(Fig["ConvBlock"]):
        channels_in: int = -1
        channels_out: int = -1
        num_convs: int = 3
        activation: Any = nn.functional.silu
        norm_momentum: float = 0.4

        def finalize(self):  # noqa: ANN201
            if self.channels_in == -1:
                self.channels_in = self.channels_out
            if self.channels_out == -1:
                self.channels_out = self.channels_in
            if self.num_convs not in (1, 2, 3):
                raise ValueError(f"num_convs must be 1, 2, or 3; got {self.num_convs}.")
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.num_convs = config.num_convs
        self.act = _activation(config.activation)
        self.pool = nn.MaxPool2d(2)
        self.convs = nn.ModuleList(
            nn.Conv2d(config.channels_in if i == 0 else config.channels_out, config.channels_out, 3, padding="same",
                      bias=False)  # fmt: skip
            for i in range(config.num_convs)
        )
        # affine-free: the next convolution absorbs any per-channel scale
        self.norms = nn.ModuleList(
            nn.BatchNorm2d(config.channels_out, eps=1e-12, momentum=config.norm_momentum, affine=False)
            for _ in range(config.num_convs)
        )

    def forward(self, x: Tensor) -> Tensor:
        x = self.act(self.norms[0](self.pool(self.convs[0](x))))
        if self.num_convs == 1:
            return x
        skip = x
        x = self.act(self.norms[1](self.convs[1](x)))
        if self.num_convs == 2:
            return x
        return self.act(self.norms[2](self.convs[2](x))) + skip


class ScaledLinear(nn.Linear):
    """Linear head whose output is multiplied by ``scale`` (default ``1 / channels_in``)."""

    class Config(Fig["ScaledLinear"]):
        channels_in: int = -1
        channels_out: int = -1
        scale: float = 0.0
        bias: bool = False

    def __init__(self, config: Config) -> None:
        super().__init__(config.channels_in, config.channels_out, bias=config.bias)
        self.scale = config.scale if config.scale > 0 else 1.0 / config.channels_in

    def forward(self, input: Tensor) -> Tensor:  # noqa: A002
        return super().forward(input) * self.scale


class ResNet(nn.Module):
    class Config(Fig["ResNet"]):
        channels_in: int = 3
        channels_hidden: tuple[int, ...] = (64, 128, 256)
        channels_out: int = 10
        block: Any = field(default_factory=ResidualBlock.Config)
        blocks_per_stage: int = 2
        activation: Any = torch.relu
        norm_momentum: float = 0.1
        proj_out: Makeable[nn.Module] | None = None

        def finalize(self):  # noqa: ANN201
            if not self.channels_hidden:
                raise ValueError("channels_hidden must name at least one stage.")
            if self.blocks_per_stage < 1:
                raise ValueError(f"blocks_per_stage must be positive; got {self.blocks_per_stage}.")
            if self.proj_out is not None:
                propagate_attr(self.proj_out, "channels_in", self.channels_hidden[-1], protocol=ChannelsIn)
                propagate_attr(self.proj_out, "channels_out", self.channels_out, protocol=ChannelsOut)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.stem = nn.Conv2d(config.channels_in, config.channels_hidden[0], 3, padding=1, bias=False)
        stages: list[nn.Module] = []
        channels = config.channels_hidden[0]
        for s, blocks in enumerate(_block_grid(config.block, len(config.channels_hidden), config.blocks_per_stage)):
            for b, block in enumerate(blocks):
                block = copy_tree(block)
                propagate_attr(block, "channels_in", channels, protocol=ChannelsIn)
                channels = config.channels_hidden[s]
                propagate_attr(block, "channels_out", channels, protocol=ChannelsOut)
                propagate_attr(block, "stride", 2 if s and not b else 1)
                propagate_attr(block, "activation", config.activation)
                propagate_attr(block, "norm_momentum", config.norm_momentum)
                stages.append(block.make())
            stages.append(nn.Identity())
        self.stages = nn.Sequential(*stages)
        self.norm = nn.BatchNorm2d(channels, momentum=config.norm_momentum)
        self.act = _activation(config.activation)
        self.pool = nn.AdaptiveAvgPool2d(1)
        self.head = config.proj_out.make() if config.proj_out is not None else nn.Linear(channels, config.channels_out)

    def forward(self, media: Tensor) -> Tensor:
        x = self.act(self.norm(self.stages(self.stem(media))))
        return self.head(self.pool(x).flatten(1))


class SpeedNet(nn.Module):
    """Whitened, wide and shallow (airbench-style); call :meth:`init_whiten` before training."""

    class Config(Fig["SpeedNet"]):
        channels_in: int = 3
        channels_hidden: tuple[int, ...] = (128, 384, 512)
        channels_out: int = 10
        block: Any = field(default_factory=ConvBlock.Config)
        whiten_kernel: int = 2
        norm_momentum: float = 0.4
        activation: Any = nn.functional.silu
        proj_out: Makeable[nn.Module] = field(default_factory=ScaledLinear.Config)
        init_conv: Any = None
        """Optional init of every block conv's leading square (``dirac``: each block starts as identity)."""

        def finalize(self):  # noqa: ANN201
            if not self.channels_hidden:
                raise ValueError("channels_hidden must name at least one block.")
            propagate_attr(self.proj_out, "channels_in", self.channels_hidden[-1], protocol=ChannelsIn)
            propagate_attr(self.proj_out, "channels_out", self.channels_out, protocol=ChannelsOut)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.whiten = PCAWhiteningConv2d(config.channels_in, config.whiten_kernel)
        self.act = _activation(config.activation)
        channels = self.whiten.out_channels
        blocks: list[nn.Module] = []
        for stage_channels, stage in zip(config.channels_hidden,
                                         _block_grid(config.block, len(config.channels_hidden), 1), strict=True):  # fmt: skip
            for block in stage:
                block = copy_tree(block)
                propagate_attr(block, "channels_in", channels, protocol=ChannelsIn)
                channels = stage_channels
                propagate_attr(block, "channels_out", channels, protocol=ChannelsOut)
                propagate_attr(block, "activation", config.activation)
                propagate_attr(block, "norm_momentum", config.norm_momentum)
                blocks.append(block.make())
        self.blocks = nn.Sequential(*blocks)
        self.pool = nn.MaxPool2d(3)
        self.head = config.proj_out.make()
        if config.init_conv is not None:
            for m in self.modules():
                if isinstance(m, nn.Conv2d) and m is not self.whiten:
                    call_init(config.init_conv, m.weight.data[: m.weight.size(1)])
            w = self.head.weight.data
            w.div_(w.std())

    def init_whiten(self, media: Tensor, *, decompose: Any = None) -> None:
        """Fit the whitening layer to a batch of training images."""
        del decompose  # symmetric eigendecomposition
        self.whiten.fit(media)

    def forward(self, media: Tensor) -> Tensor:
        return self.head(self.pool(self.blocks(self.act(self.whiten(media)))).flatten(1))
