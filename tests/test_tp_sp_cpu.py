"""Fused sequence-parallel TP: sharding, gradient reductions and clipping on gloo ranks.

On CPU the layers run the torch.distributed oracle communicator with the same
row layout, head/gate slicing, gradient hooks and TP-aware clip norm as the
fused NVLink kernels.
"""

from __future__ import annotations

import torch

from priml_b200.testing import run_ranks


def _cfg(parallelism, clip: float = 1.0):  # noqa: ANN001, ANN202
    from priml_b200.loss import TokenCrossEntropy
    from priml_b200.models.presets import tiny_lm
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.train import TrainStep

    return TrainStep.Config(
        model=tiny_lm(),
        optimizer=FusedAdamW.Config(lr=3e-3, betas=(0.9, 0.95), weight_decay=0.1),
        loss=TokenCrossEntropy.Config(),
        parallelism=parallelism,
        gradient_clip_norm=clip,
    )


def _batches(n: int) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 512, (8, 33), generator=g) for _ in range(n)]


def _tp(rank: int, world: int, steps: int, accumulate: int = 1) -> dict:
    from priml_b200.parallel.tp_fused import FusedSequenceParallel, SPColumnLinear

    torch.manual_seed(0)
    cfg = _cfg(FusedSequenceParallel.Config())
    cfg.accumulate_grad_batches = accumulate
    step = cfg.make()
    losses, norms = [], []
    for seq in _batches(steps):
        local = seq.chunk(world)[rank]
        for micro in local.chunk(accumulate):
            out = step.train_step(tokens=micro[:, :-1], targets=micro[:, 1:])
        t = out["loss"].detach().float().mean()
        if world > 1:
            torch.distributed.all_reduce(t)
        losses.append(float(t) / world)
        norms.append(float(step.last_grad_norm))
    shapes = {n: tuple(p.shape) for n, p in step.model.named_parameters()}
    cols = sum(isinstance(m, SPColumnLinear) for m in step.model.modules())
    return {"losses": losses, "norms": norms, "shapes": shapes, "cols": cols}


def _single(steps: int) -> dict:
    torch.manual_seed(0)
    step = _cfg(None).make()
    losses, norms = [], []
    for seq in _batches(steps):
        out = step.train_step(tokens=seq[:, :-1], targets=seq[:, 1:])
        losses.append(float(out["loss"].float().mean()))
        norms.append(float(step.last_grad_norm))
    return {"losses": losses, "norms": norms}


def test_tp2_matches_single_process() -> None:
    ref = _single(4)
    two = run_ranks(_tp, 2, 4, mesh_shape={"tp": 2})
    assert two[0]["losses"] == two[1]["losses"]
    assert two[0]["cols"] == 4  # qkv + up per block, 2 blocks
    # heads and hidden units split in half
    qkv = [s for n, s in two[0]["shapes"].items() if n.endswith("proj_qkv.weight")]
    assert qkv and qkv[0][0] == 6, qkv  # (4 q + 4 k + 4 v heads) / 2
    for a, b in zip(two[0]["losses"], ref["losses"], strict=True):
        assert abs(a - b) < 2e-3 * max(1.0, abs(b)), (two[0]["losses"], ref["losses"])
    for a, b in zip(two[0]["norms"], ref["norms"], strict=True):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (two[0]["norms"], ref["norms"])


def test_tp2_gradient_accumulation_matches_full_batch() -> None:
    full = run_ranks(_tp, 2, 3, 1, mesh_shape={"tp": 2})
    acc = run_ranks(_tp, 2, 3, 2, mesh_shape={"tp": 2})
    for a, b in zip(acc[0]["norms"], full[0]["norms"], strict=True):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (acc[0]["norms"], full[0]["norms"])


def test_dp2_tp2_matches_single_process() -> None:
    ref = _single(3)
    four = run_ranks(_tp, 4, 3, mesh_shape={"dp": 2, "tp": 2})
    for a, b in zip(four[0]["losses"], ref["losses"], strict=True):
        assert abs(a - b) < 2e-3 * max(1.0, abs(b)), (four[0]["losses"], ref["losses"])
    for a, b in zip(four[0]["norms"], ref["norms"], strict=True):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (four[0]["norms"], ref["norms"])
