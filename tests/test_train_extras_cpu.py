"""GAN step, eval/train loss paths, protocols, progress and results files."""

from __future__ import annotations

import json

import torch
from torch import nn

from priml_b200.config import InlineConfig


class _Gen(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.net = nn.Linear(4, 6)

    def forward(self, noise: torch.Tensor, **kwargs) -> torch.Tensor:  # noqa: ANN003
        del kwargs
        return torch.tanh(self.net(noise))

    def reset_parameters(self) -> None:
        self.net.reset_parameters()


class _Disc(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.net = nn.Sequential(nn.Linear(6, 8), nn.ReLU(), nn.Linear(8, 1))
        self.frozen = nn.Parameter(torch.ones(1), requires_grad=False)

    def forward(self, media: torch.Tensor) -> torch.Tensor:
        return self.net(media) * self.frozen

    def reset_parameters(self) -> None:
        for m in self.net:
            if hasattr(m, "reset_parameters"):
                m.reset_parameters()


def test_gan_step_updates_both_players_and_keeps_frozen_flags() -> None:
    from priml_b200.train import GANTrainStep, TrainStep

    torch.manual_seed(0)
    cfg = GANTrainStep.Config(n_discriminator_steps=2)
    cfg.generator.model = InlineConfig(_Gen)
    cfg.discriminator.model = InlineConfig(_Disc)
    gan = cfg.make()
    assert isinstance(gan.generator, TrainStep)
    g0 = gan.generator.model.net.weight.detach().clone()
    d0 = gan.discriminator.model.net[0].weight.detach().clone()
    real = torch.rand(5, 6) * 2 - 1
    out = gan.train_step(media=real, noise=torch.randn(5, 4))
    assert out["loss"].shape == (5,) and out["model"].shape == (5, 6)
    assert not torch.equal(g0, gan.generator.model.net.weight)
    assert not torch.equal(d0, gan.discriminator.model.net[0].weight)
    assert gan.discriminator.model.frozen.requires_grad is False
    assert all(p.requires_grad for p in gan.discriminator.model.net.parameters())
    assert gan.global_step == 1
    ev = gan.eval_loss(media=real, noise=torch.randn(5, 4))
    tl = gan.train_loss(media=real, noise=torch.randn(5, 4))
    assert ev["loss"].shape == (5,) and tl["loss"].shape == (5,)
    sd = gan.state_dict()
    gan.load_state_dict(sd)
    assert gan.global_step == 1 and gan.local_step == 0


def test_lm_eval_loss_and_call_eval() -> None:
    from priml_b200.loss import TokenCrossEntropy
    from priml_b200.models.presets import tiny_lm
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.train import TrainStep

    torch.manual_seed(0)
    step = TrainStep.Config(model=tiny_lm(), optimizer=FusedAdamW.Config(), loss=TokenCrossEntropy.Config()).make()
    seq = torch.randint(0, 512, (2, 17))
    ev = step.eval_loss(tokens=seq[:, :-1], targets=seq[:, 1:])
    tr = step.train_loss(tokens=seq[:, :-1], targets=seq[:, 1:])
    assert torch.allclose(ev["loss"], tr["loss"])
    logits = step.call_eval(tokens=seq[:, :-1])
    assert logits.shape == (2, 16, 512) and step.model.training


def test_protocols_progress_and_results(tmp_path) -> None:  # noqa: ANN001
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.train import EMA, Checkpointer, NoEMA, format_summary, read_metrics, summarize, write_progress
    from priml_b200.train.custom_types import CheckpointableProtocol, EMAProtocol, OptimizerProtocol

    opt = FusedAdamW([nn.Parameter(torch.zeros(3))])
    assert isinstance(opt, OptimizerProtocol) and isinstance(opt, CheckpointableProtocol)
    assert isinstance(NoEMA(), EMAProtocol)
    del EMA, Checkpointer
    p = write_progress(3, 10, working_dir=tmp_path, metrics={"loss": 1.5})
    data = json.loads(p.read_text())
    assert data["step"] == 3 and data["total"] == 10 and data["metrics"] == {"loss": 1.5}
    assert not list(tmp_path.glob("*.tmp"))
    m = tmp_path / "metrics.json"
    m.write_text(json.dumps({"eval/loss": 2.0, "eval/acc": 0.5}))
    assert read_metrics(m) == {"eval/loss": 2.0, "eval/acc": 0.5}
    assert format_summary(read_metrics(m)) == "acc=0.5 loss=2.0"
    assert format_summary(read_metrics(m), ["eval/loss"]) == "loss=2.0"
    assert summarize(["--path", str(m)]) == 0
    assert summarize(["--path", str(tmp_path / "missing.json")]) == 1


def test_augmentation_torch_path() -> None:
    from priml_b200.data.augmentation_gpu import AugmentDraws, cutout, flip_lr, pad_crop_flip, random_crop

    torch.manual_seed(0)
    img = torch.arange(2 * 3 * 6 * 6, dtype=torch.float32).reshape(2, 3, 6, 6)
    z = torch.zeros(2, dtype=torch.int32)
    ident = AugmentDraws(z + 2, z + 2, None, z, z)
    assert torch.equal(pad_crop_flip(img, 6, pad=2, draws=ident), img)
    flipped = AugmentDraws(z + 2, z + 2, torch.ones(2, dtype=torch.uint8), z, z)
    assert torch.equal(pad_crop_flip(img, 6, pad=2, draws=flipped), img.flip(-1))
    shifted = AugmentDraws(z, z, None, z, z)
    out = pad_crop_flip(img, 6, pad=2, pad_mode="constant", draws=shifted)
    assert torch.equal(out[..., 2:, 2:], img[..., :4, :4]) and float(out[..., :2, :].abs().sum()) == 0.0
    cut = AugmentDraws(z + 2, z + 2, None, z + 1, z + 2)
    c = pad_crop_flip(img, 6, pad=2, cutout_size=3, draws=cut)
    assert float(c[:, :, 1:4, 2:5].abs().sum()) == 0.0 and torch.equal(c[:, :, 0], img[:, :, 0])
    rnd = pad_crop_flip(torch.rand(8, 3, 32, 32), 32, pad=4, cutout_size=8)
    assert rnd.shape == (8, 3, 32, 32) and rnd.is_contiguous()
    assert random_crop(torch.rand(4, 3, 10, 10), 8).shape == (4, 3, 8, 8)
    assert flip_lr(img).shape == img.shape and cutout(img, 2).shape == img.shape
