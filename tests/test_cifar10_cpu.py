"""CIFAR-10 baseline: networks, whitening, augmentation, schedule, TTA and the loop (CPU, synthetic images)."""

from __future__ import annotations

from pathlib import Path

import torch


def _prepared(tmp_path: Path) -> Path:
    from priml_b200.baselines.cifar10.data import prepare_from_arrays

    g = torch.Generator().manual_seed(0)
    for split, n in (("train", 256), ("test", 64)):
        labels = torch.randint(0, 10, (n,), generator=g)
        # class-dependent colour so a few steps can learn something
        base = (labels.view(n, 1, 1, 1).float() * 25).expand(n, 32, 32, 3)
        images = (base + torch.randint(0, 40, (n, 32, 32, 3), generator=g)).clamp(0, 255).to(torch.uint8)
        prepare_from_arrays(tmp_path, split, images, labels)
    return tmp_path


def test_networks_shapes_and_whitening() -> None:
    from priml_b200.baselines.cifar10 import ResNet, SpeedNet

    x = torch.randn(8, 3, 32, 32)
    r = ResNet.Config(channels_hidden=(8, 16), blocks_per_stage=1).make()
    assert r(x).shape == (8, 10)
    s = SpeedNet.Config(channels_hidden=(16, 24, 32)).make()
    s.init_whiten(x)
    w = s.whiten(x)
    assert w.shape[1] == 24  # 2 * 3 * 2 * 2 whitening filters
    assert s(x).shape == (8, 10)
    assert not s.whiten.weight.requires_grad


def test_speednet_muon_tta_loop_trains(tmp_path: Path) -> None:
    from priml_b200.baselines.cifar10.experiments import exp004

    cfg = exp004()
    cfg.working_dir = str(tmp_path / "run")
    cfg.dataset.working_dir = str(_prepared(tmp_path))
    cfg.dataset.device = "cpu"
    cfg.dataset.batch_size = 64
    cfg.dataset.eval_batch_size = 64
    cfg.step.model.channels_hidden = (16, 32, 32)
    cfg.max_steps = cfg.step.total_train_steps = 12
    cfg.num_steps_eval = 6
    cfg.step.whiten_cache_path = str(tmp_path / "whiten.pt")
    loop = cfg.make()
    res = loop.train()
    assert loop.global_step == 12
    assert 0.0 <= res["eval/accuracy_top1"] <= 1.0
    assert (tmp_path / "whiten.pt").is_file()
    assert loop.step.state_dict()["whitened"] is True


def test_resnet_adamw_schedule_warms_up(tmp_path: Path) -> None:
    from priml_b200.baselines.cifar10.experiments import exp000

    cfg = exp000()
    cfg.working_dir = str(tmp_path / "run")
    cfg.dataset.working_dir = str(_prepared(tmp_path))
    cfg.dataset.device = "cpu"
    cfg.dataset.batch_size = 64
    cfg.step.model.channels_hidden = (8, 16)
    cfg.step.model.blocks_per_stage = 1
    cfg.max_steps = cfg.step.total_train_steps = 100
    cfg.step.warmup_fraction = 0.05
    loop = cfg.make()
    step = loop.step
    it = iter(loop.dataset.train_dataloader())
    lrs = []
    for _ in range(3):
        step.train_step(**next(it))
        lrs.append(step.optimizer.param_groups[0]["lr"])
    # warmup of int(0.05 * 100) = 5 whole steps, reading one step ahead
    assert lrs[0] < lrs[1] < lrs[2] <= 1e-3
    assert abs(lrs[0] - 1e-3 * 1 / 5 * 1.0) < 1e-5
