"""Baselines on the GPU: nanochat (windowed tcgen05 attention, value gates, fused soft-capped loss)
and CIFAR-10 SpeedNet (fused augmentation, channels-last bf16)."""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_nanochat_trains_on_cuda() -> None:
    from priml_b200.baselines.nanochat.experiments import exp000
    from priml_b200.ops import native

    torch.manual_seed(0)
    cfg = exp000().step
    cfg.model.num_layers = 4
    cfg.model.max_seq_len = 512
    cfg.rows_per_pass = 8
    cfg.tokens_per_optimizer_step = 8 * 512
    cfg.budget_warmup_steps = 0
    step = cfg.make()
    g = torch.Generator(device="cuda").manual_seed(1)
    seq = torch.randint(0, 64, (8, 513), device="cuda", generator=g)  # a small effective vocabulary: learnable
    losses = []
    for _ in range(6):
        out = step.train_step(media=seq[:, :-1], label=seq[:, 1:])
        losses.append(float(out["loss"]))
    assert all(math.isfinite(x) for x in losses) and losses[-1] < losses[0], losses
    # the fused loss equals the logits path on the device
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused = step.model.token_loss(seq[:, :-1], seq[:, 1:])
        logits = step.model(seq[:, :-1])
    ref = torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), seq[:, 1:].reshape(-1),
                                            reduction="none").view(8, 512)  # fmt: skip
    assert float((fused - ref).abs().max()) < 2e-2
    assert int(native().read_status(True)) == 0


def test_cifar10_speednet_trains_on_cuda(tmp_path) -> None:  # noqa: ANN001
    from priml_b200.baselines.cifar10.data import prepare_from_arrays
    from priml_b200.baselines.cifar10.experiments import exp003

    g = torch.Generator().manual_seed(0)
    for split, n in (("train", 2048), ("test", 512)):
        labels = torch.randint(0, 10, (n,), generator=g)
        base = (labels.view(n, 1, 1, 1).float() * 25).expand(n, 32, 32, 3)
        images = (base + torch.randint(0, 40, (n, 32, 32, 3), generator=g)).clamp(0, 255).to(torch.uint8)
        prepare_from_arrays(tmp_path, split, images, labels)
    cfg = exp003()
    cfg.working_dir = str(tmp_path / "run")
    cfg.dataset.working_dir = str(tmp_path)
    cfg.dataset.batch_size = 256
    cfg.dataset.eval_batch_size = 512
    cfg.step.dtype_autocast = torch.bfloat16
    cfg.max_steps = cfg.step.total_train_steps = 24
    cfg.num_steps_eval = 24
    loop = cfg.make()
    res = loop.train()
    assert res["eval/accuracy_top1"] > 0.5, res  # colour-coded classes are easy


def test_sudoku_recurrent_step_on_cuda(monkeypatch) -> None:  # noqa: ANN001
    """The recurrent rung (6 x 9 cycles, ACT pool, feedback) on the tcgen05 kernels: the
    bidirectional 81-token attention and the GEMMs agree with the torch oracle, and a few
    steps of training reduce the loss."""
    from priml_b200.baselines.sudoku.act import ActPool
    from priml_b200.baselines.sudoku.experiments import exp002
    from priml_b200.ops import native

    cfg = exp002().step
    cfg.act = ActPool.Config(batch_size=64, max_steps=4)
    cfg.model.recurrence.slow_cycles = 2
    cfg.model.recurrence.fast_cycles = 3
    torch.manual_seed(0)
    step = cfg.make()
    g = torch.Generator(device="cuda").manual_seed(0)
    label = torch.randint(2, 11, (64, 81), device="cuda", generator=g)
    media = torch.where(torch.rand(64, 81, device="cuda", generator=g) < 0.5, label, torch.ones_like(label))
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        z = step.model.init_latents(64)
        fast = step.model(media, *z).logits.float()
        monkeypatch.setenv("PRIML_B200_REFERENCE", "1")
        ref = step.model(media, *z).logits.float()
        monkeypatch.delenv("PRIML_B200_REFERENCE")
    assert float((fast - ref).abs().max() / ref.abs().max()) < 5e-2
    losses = [float(step.train_step(media=media, label=label, valid_count=64)["lm_loss"]) for _ in range(8)]
    assert all(math.isfinite(x) for x in losses) and losses[-1] < losses[0], losses
    out = step.eval_loss(media=media, label=label, valid_count=64)
    assert out["model"].shape == (64, 82)
    assert int(native().read_status(True)) == 0


def test_arc_transformer_step_on_cuda(monkeypatch) -> None:  # noqa: ANN001
    """The ARC exp000 solver at full width: 917-token bidirectional attention (16 puzzle tokens +
    1 register + 900 cells) on the tcgen05 kernels against the torch oracle, then training steps
    with the sparse per-puzzle table stepped by sign-SGD."""
    from priml_b200.baselines.arcagi1.experiments import exp000
    from priml_b200.ops import native
    from priml_b200.optimizers import SignSGD

    cfg = exp000().step
    cfg.model.prefix.parts[0].num_puzzles = 32
    cfg.model.prefix.parts[0].batch_size = 8
    cfg.puzzle_optimizer = SignSGD.Config(lr=0.01)
    torch.manual_seed(0)
    step = cfg.make()
    g = torch.Generator(device="cuda").manual_seed(0)
    media = torch.randint(0, 12, (8, 900), device="cuda", generator=g)
    label = torch.where(media >= 2, 13 - media, media)  # a fixed recoloring rule
    ids = torch.arange(8, device="cuda") * 3
    step.model.eval()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fast = step.model(media, puzzle_identifiers=ids).logits.float()
        monkeypatch.setenv("PRIML_B200_REFERENCE", "1")
        ref = step.model(media, puzzle_identifiers=ids).logits.float()
        monkeypatch.delenv("PRIML_B200_REFERENCE")
    assert float((fast - ref).abs().max() / ref.abs().max()) < 5e-2
    losses = [float(step.train_step(media=media, label=label, valid_count=8, puzzle_identifiers=ids)["lm_loss"])
              for _ in range(6)]  # fmt: skip
    assert all(math.isfinite(x) for x in losses) and losses[-1] < losses[0], losses
    table = step.model.prefix.parts[0].weights
    assert float(table[ids].abs().sum()) > 0 and float(table[1].abs().sum()) == 0
    assert int(native().read_status(True)) == 0


def test_craftax_ppo_update_on_cuda() -> None:
    """The batched game, the 8,268-wide observation and a PPO update (bf16 tcgen05 GEMMs) on the device."""
    from priml_b200.baselines.craftax import CraftaxEnv, CraftaxTrainStep
    from priml_b200.ops import native

    cfg = CraftaxTrainStep.Config()
    cfg.env = CraftaxEnv.Config(num_envs=256, device="cuda", seed=0)
    cfg.rollout_steps = 16
    step = cfg.make()
    assert step.env.device.type == "cuda"
    out = [step.train_step() for _ in range(2)]
    assert all(bool(torch.isfinite(o["loss"]).all()) for o in out)
    assert math.isfinite(float(out[-1]["metrics"]["explained_variance"]))
    assert int(native().read_status(True)) == 0
