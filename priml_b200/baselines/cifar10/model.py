"""CIFAR-10 networks (``priml/baselines/cifar10/model.py:40-558``).

* ``ResNet``: pre-activation residual stages (norm, activation, conv), a
  stride-2 first block per later stage, global average pool, linear head.
* ``SpeedNet``: the speedrun design -- a frozen PCA patch-whitening conv fitted
  on training images, then wide ``ConvBlock`` stages (conv, max-pool, affine-free
  batch norm, activation; a residual over the last two convs), max-pool, and a
  head scaled by ``1 / channels``.

Module and parameter names (``stem``, ``stages.{i}``, ``norm``, ``head``,
``whiten``, ``blocks.{i}.convs.{j}``, ``norm1`` / ``conv1`` / ``norm2`` / ``conv2`` /
``shortcut``) are the reference's, so checkpoints load in either framework.
Each network is built from a *plan*: the list of (block config, input width,
output width, stride) it instantiates, computed once from the config.

Convolutions run channels-last in bf16 under autocast through cuDNN (library
convolutions; the network's hot path is small 3x3 convs that cuDNN's sm_100
kernels already cover).
"""

from __future__ import annotations

from dataclasses import field
from typing import Any, NamedTuple

import torch
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable, copy_tree
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, propagate_attr
from priml_b200.models.init import call_init
from priml_b200.models.vision import PCAWhiteningConv2d

__all__ = ["ConvBlock", "ResNet", "ResidualBlock", "ScaledLinear", "SpeedNet"]


def _activation(act: Any) -> Any:
    """A config of an activation module is made; a plain callable is used as is."""
    return act.make() if hasattr(act, "make") else act


def _fill_widths(cfg: Any) -> None:
    """A block given only one of its widths keeps the width unchanged."""
    if cfg.channels_in == -1:
        cfg.channels_in = cfg.channels_out
    elif cfg.channels_out == -1:
        cfg.channels_out = cfg.channels_in


class _Step(NamedTuple):
    """One block of a network plan."""

    template: Any
    c_in: int
    c_out: int
    stride: int
    stage: int
    last_in_stage: bool


def _plan(block: Any, widths: tuple[int, ...], per_stage: int, c_start: int, *, downsample: bool) -> list[_Step]:
    """The blocks of ``len(widths)`` stages of ``per_stage`` blocks each, chained by width.

    ``block`` is one template copied for every slot, or an explicit flat list with one config
    per slot. With ``downsample`` the first block of every stage after the first halves the
    resolution (the first stage keeps the full 32 x 32 grid).
    """
    slots = len(widths) * per_stage
    if isinstance(block, list):
        if len(block) != slots:
            raise ValueError(f"{len(widths)} stages x {per_stage} blocks need {slots} block configs, not {len(block)}.")
        templates = list(block)
    else:
        templates = [block] * slots
    steps, c_prev = [], c_start
    for i, template in enumerate(templates):
        stage, pos = divmod(i, per_stage)
        stride = 2 if downsample and stage > 0 and pos == 0 else 1
        steps.append(_Step(template, c_prev, widths[stage], stride, stage, pos == per_stage - 1))
        c_prev = widths[stage]
    return steps


def _make_block(step: _Step, **shared: Any) -> nn.Module:
    cfg = copy_tree(step.template)
    propagate_attr(cfg, "channels_in", step.c_in, protocol=ChannelsIn)
    propagate_attr(cfg, "channels_out", step.c_out, protocol=ChannelsOut)
    for name, value in shared.items():
        propagate_attr(cfg, name, value)
    return cfg.make()


class ResidualBlock(nn.Module):
    """Pre-activation residual block; the skip is projected by a 1x1 conv when the shape changes."""

    class Config(Fig["ResidualBlock"]):
        channels_in: int = -1
        channels_out: int = -1
        stride: int = 1
        activation: Any = torch.relu
        norm_momentum: float = 0.1

        def finalize(self):  # noqa: ANN201
            _fill_widths(self)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        c_in, c_out, stride = config.channels_in, config.channels_out, config.stride

        def conv(a: int, b: int, k: int, s: int = 1) -> nn.Conv2d:
            return nn.Conv2d(a, b, k, stride=s, padding=k // 2, bias=False)

        self.norm1 = nn.BatchNorm2d(c_in, momentum=config.norm_momentum)
        self.conv1 = conv(c_in, c_out, 3, stride)
        self.norm2 = nn.BatchNorm2d(c_out, momentum=config.norm_momentum)
        self.conv2 = conv(c_out, c_out, 3)
        self.act = _activation(config.activation)
        reshapes = stride != 1 or c_in != c_out
        self.shortcut = conv(c_in, c_out, 1, stride) if reshapes else nn.Identity()

    def forward(self, x: Tensor) -> Tensor:
        # Both paths start from the normalized, activated input: projecting raw activations
        # in the skip diverges in deep stacks.
        pre = self.act(self.norm1(x))
        branch = self.conv2(self.act(self.norm2(self.conv1(pre))))
        return branch + self.shortcut(pre)


class ConvBlock(nn.Module):
    """conv -> max-pool -> norm -> act, then up to two more conv -> norm -> act layers.

    With three convolutions the output of the first layer is added back after the third.
    The norms have no affine parameters: the next convolution absorbs any channel scale.
    """

    class Config(Fig["ConvBlock"]):
        channels_in: int = -1
        channels_out: int = -1
        num_convs: int = 3
        activation: Any = nn.functional.silu
        norm_momentum: float = 0.4

        def finalize(self):  # noqa: ANN201
            _fill_widths(self)
            if not 1 <= self.num_convs <= 3:
                raise ValueError(f"ConvBlock has one, two or three convolutions; num_convs={self.num_convs}.")
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        widths = [config.channels_in] + [config.channels_out] * config.num_convs
        self.num_convs = config.num_convs
        self.act = _activation(config.activation)
        self.pool = nn.MaxPool2d(2)
        self.convs = nn.ModuleList(
            [nn.Conv2d(a, b, 3, padding="same", bias=False) for a, b in zip(widths[:-1], widths[1:], strict=True)]
        )
        self.norms = nn.ModuleList(
            [
                nn.BatchNorm2d(config.channels_out, eps=1e-12, momentum=config.norm_momentum, affine=False)
                for _ in range(config.num_convs)
            ]
        )

    def forward(self, x: Tensor) -> Tensor:
        first = None
        for i, (conv, norm) in enumerate(zip(self.convs, self.norms, strict=True)):
            y = conv(x)
            if i == 0:
                y = self.pool(y)
            x = self.act(norm(y))
            if i == 0:
                first = x
            elif i == 2:
                x = x + first
        return x


class ScaledLinear(nn.Linear):
    """Linear head whose output is multiplied by ``scale`` (default ``1 / channels_in``)."""

    class Config(Fig["ScaledLinear"]):
        channels_in: int = -1
        channels_out: int = -1
        scale: float = 0.0
        bias: bool = False

    def __init__(self, config: Config) -> None:
        super().__init__(config.channels_in, config.channels_out, bias=config.bias)
        self.scale = 1.0 / config.channels_in if config.scale <= 0 else config.scale

    def forward(self, input: Tensor) -> Tensor:  # noqa: A002
        return torch.mul(nn.functional.linear(input, self.weight, self.bias), self.scale)


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
            if len(self.channels_hidden) == 0:
                raise ValueError("ResNet needs at least one stage width in channels_hidden.")
            if self.blocks_per_stage <= 0:
                raise ValueError(f"ResNet needs at least one block per stage; blocks_per_stage={self.blocks_per_stage}.")
            if self.proj_out is not None:
                propagate_attr(self.proj_out, "channels_in", self.channels_hidden[-1], protocol=ChannelsIn)
                propagate_attr(self.proj_out, "channels_out", self.channels_out, protocol=ChannelsOut)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        widths = tuple(config.channels_hidden)
        self.stem = nn.Conv2d(config.channels_in, widths[0], 3, padding=1, bias=False)
        layers: list[nn.Module] = []
        for step in _plan(config.block, widths, config.blocks_per_stage, widths[0], downsample=True):
            layers.append(_make_block(step, stride=step.stride, activation=config.activation,
                                      norm_momentum=config.norm_momentum))  # fmt: skip
            if step.last_in_stage:
                layers.append(nn.Identity())  # stage boundary; keeps the checkpoint's module indices
        self.stages = nn.Sequential(*layers)
        self.norm = nn.BatchNorm2d(widths[-1], momentum=config.norm_momentum)
        self.act = _activation(config.activation)
        self.pool = nn.AdaptiveAvgPool2d(1)
        self.head = nn.Linear(widths[-1], config.channels_out) if config.proj_out is None else config.proj_out.make()

    def forward(self, media: Tensor) -> Tensor:
        features = self.act(self.norm(self.stages(self.stem(media))))
        return self.head(torch.flatten(self.pool(features), 1))


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
            if len(self.channels_hidden) == 0:
                raise ValueError("SpeedNet needs at least one block width in channels_hidden.")
            propagate_attr(self.proj_out, "channels_in", self.channels_hidden[-1], protocol=ChannelsIn)
            propagate_attr(self.proj_out, "channels_out", self.channels_out, protocol=ChannelsOut)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.whiten = PCAWhiteningConv2d(config.channels_in, config.whiten_kernel)
        self.act = _activation(config.activation)
        steps = _plan(config.block, tuple(config.channels_hidden), 1, self.whiten.out_channels, downsample=False)
        self.blocks = nn.Sequential(
            *[_make_block(s, activation=config.activation, norm_momentum=config.norm_momentum) for s in steps]
        )
        self.pool = nn.MaxPool2d(3)
        self.head = config.proj_out.make()
        if config.init_conv is not None:
            self._init_convs(config.init_conv)

    def _init_convs(self, init: Any) -> None:
        """Apply ``init`` to the square leading slice of every block conv; unit-variance head."""
        convs = [m for m in self.blocks.modules() if isinstance(m, nn.Conv2d)]
        for conv in convs:
            square = conv.weight.data.narrow(0, 0, min(conv.weight.size(0), conv.weight.size(1)))
            call_init(init, square)
        head = self.head.weight.data
        head.mul_(1.0 / head.std())

    def init_whiten(self, media: Tensor, *, decompose: Any = None) -> None:
        """Fit the whitening layer to a batch of training images."""
        del decompose  # symmetric eigendecomposition
        self.whiten.fit(media)

    def forward(self, media: Tensor) -> Tensor:
        features = self.blocks(self.act(self.whiten(media)))
        return self.head(torch.flatten(self.pool(features), 1))
