"""CIFAR-10 image classification (``priml/baselines/cifar10``)."""

from priml_b200.baselines.cifar10.model import ConvBlock, ResidualBlock, ResNet, ScaledLinear, SpeedNet
from priml_b200.baselines.cifar10.train_step import Cifar10TrainStep, tta_logits

__all__ = ["Cifar10TrainStep", "ConvBlock", "ResNet", "ResidualBlock", "ScaledLinear", "SpeedNet", "tta_logits"]
