"""CIFAR-10 experiment ladder (``priml/baselines/cifar10/experiments.py``).

* ``exp000``: pre-activation ResNet, AdamW, cosine, crops + flips, 30 epochs.
* ``exp001``: exp000 with SpeedNet (PCA whitening, wide and shallow), 8 epochs.
* ``exp002``: exp001 with Muon on the convolutions and Nesterov SGD on the rest,
  polynomial (power 1.2) decay.
* ``exp003``: exp002 with test-time augmentation.
* ``exp004``: exp003 with dirac-initialized convolutions, cutout and derandomized flips.
"""

from __future__ import annotations

from dataclasses import field
from typing import Any, Final

import torch

from priml_b200.baselines.cifar10.data import Cifar10Data
from priml_b200.baselines.cifar10.model import ResNet, SpeedNet
from priml_b200.baselines.cifar10.train_step import Cifar10TrainStep
from priml_b200.config import Makes, PartialConfig
from priml_b200.math.schedules import polynomial
from priml_b200.metrics import TopK
from priml_b200.models.init import dirac
from priml_b200.optimizers.composite import CompositeOptimizer, complement, excluding
from priml_b200.optimizers.muon import Muon, adjust_lr_conv_heuristic
from priml_b200.parallel.runtime import SingleProcess
from priml_b200.train.train_loop import TrainLoop

__all__ = ["Cifar10TrainLoop", "NUM_TRAIN_SAMPLES", "exp000", "exp001", "exp002", "exp003", "exp004"]

NUM_TRAIN_SAMPLES: Final = 50_000


class Cifar10TrainLoop(Makes["TrainLoop"], TrainLoop.Config):
    step: Any = field(default_factory=Cifar10TrainStep.Config)
    dataset: Any = field(default_factory=Cifar10Data.Config)


def exp000() -> Cifar10TrainLoop:
    cfg = Cifar10TrainLoop()
    cfg.study_name = "cifar10"
    cfg.experiment_name = "exp000"
    cfg.step.model = ResNet.Config()
    cfg.dataset.batch_size = 512
    per_epoch = NUM_TRAIN_SAMPLES // cfg.dataset.batch_size
    cfg.num_steps_eval = per_epoch
    cfg.max_steps = cfg.step.total_train_steps = 30 * per_epoch
    cfg.metrics["accuracy"] = TopK.Config(k_values=[1])
    cfg.runtime = SingleProcess.Config()
    return cfg


def exp001() -> Cifar10TrainLoop:
    cfg = exp000()
    cfg.experiment_name = "exp001"
    cfg.step.model = SpeedNet.Config()
    cfg.max_steps = cfg.step.total_train_steps = 8 * (NUM_TRAIN_SAMPLES // cfg.dataset.batch_size)
    return cfg


def exp002() -> Cifar10TrainLoop:
    cfg = exp001()
    cfg.experiment_name = "exp002"
    on_muon = excluding(Muon.eligible_tensor, "head")
    split = CompositeOptimizer.Config()
    split.select = [complement(on_muon), on_muon]
    sgd = PartialConfig(torch.optim.SGD, lr=0.67, momentum=0.85, nesterov=True)
    muon = Muon.Config(lr=0.24, momentum=0.6, nesterov=True, ns_steps=3, weight_decay=0.0125,
                       adjust_lr_fn=adjust_lr_conv_heuristic)  # fmt: skip
    split.optimizers = [sgd, muon]
    cfg.step.optimizer = split
    cfg.step.schedule = PartialConfig(polynomial, power=1.2)
    return cfg


def exp003() -> Cifar10TrainLoop:
    cfg = exp002()
    cfg.experiment_name = "exp003"
    cfg.step.use_tta = True
    return cfg


def exp004() -> Cifar10TrainLoop:
    cfg = exp003()
    cfg.experiment_name = "exp004"
    cfg.step.model.init_conv = dirac
    cfg.step.cutout_size = 12
    cfg.step.derandomized_flip = True
    return cfg
