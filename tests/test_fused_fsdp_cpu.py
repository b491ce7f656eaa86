"""Sharded data parallelism with fused collectives: host-side plumbing on gloo ranks.

On CPU the strategy runs its torch.distributed oracle path (all-reduce +
all-gather) with the same flat layout, buckets, gradient sinks, readiness
hooks, shard segments and checkpoint hooks as the CUDA kernels use.
"""

from __future__ import annotations

import pytest
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
    return [torch.randint(0, 512, (8, 65), generator=g) for _ in range(n)]


def _sharded(rank: int, world: int, steps: int, accumulate: int = 1, shard_params: bool = False) -> dict:
    from priml_b200.parallel.fused_fsdp import FusedFullySharded

    torch.manual_seed(0)
    cfg = _cfg(FusedFullySharded.Config(device="cpu", shard_params=shard_params))
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
    sd = step.model.state_dict()
    osd = step.optimizer.state_dict()
    return {
        "losses": losses,
        "norms": norms,
        "dtypes": sorted({str(v.dtype) for v in sd.values()}),
        "keys": sorted(sd),
        "opt_keys": sorted(osd["state"][0]),
        "weights": {k: v.clone() for k, v in sd.items()},
        "shard_elems": step.parallelism.state.param_buf.numel(),
        "total_elems": step.parallelism.state.total,
    }


def test_sharded_world2_matches_world1() -> None:
    one = run_ranks(_sharded, 1, 4)[0]
    two = run_ranks(_sharded, 2, 4, mesh_shape={"dp": 2})
    assert two[0]["losses"] == two[1]["losses"]
    for a, b in zip(two[0]["losses"], one["losses"], strict=True):
        assert abs(a - b) < 5e-3 * max(1.0, abs(b)), (a, b)
    for a, b in zip(two[0]["norms"], one["norms"], strict=True):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), (a, b)
    # every rank reconstructs the same fp32 master weights for checkpoints
    for k, v in two[0]["weights"].items():
        assert torch.equal(v, two[1]["weights"][k])
    assert two[0]["dtypes"] == ["torch.float32"]
    assert two[0]["opt_keys"] == ["first_moment", "second_moment", "step"]


def test_sharded_tracks_unsharded_fused_adamw() -> None:
    one = run_ranks(_sharded, 1, 4)[0]
    torch.manual_seed(0)
    ref = _cfg(None).make()
    ref_losses = []
    for seq in _batches(4):
        with torch.autocast("cpu", dtype=torch.bfloat16):
            out = ref.train_step(tokens=seq[:, :-1], targets=seq[:, 1:])
        ref_losses.append(float(out["loss"].float().mean()))
    assert sorted(one["keys"]) == sorted(ref.model.state_dict())
    for a, b in zip(one["losses"], ref_losses, strict=True):
        assert abs(a - b) < 3e-2 * max(1.0, abs(b)), (one["losses"], ref_losses)


def test_sharded_gradient_accumulation_matches_full_batch() -> None:
    full = run_ranks(_sharded, 2, 3, 1, mesh_shape={"dp": 2})
    acc = run_ranks(_sharded, 2, 3, 2, mesh_shape={"dp": 2})
    assert abs(full[0]["losses"][0] - 0.0) > 0
    for a, b in zip(acc[0]["norms"], full[0]["norms"], strict=True):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), (acc[0]["norms"], full[0]["norms"])


def _resume(rank: int, world: int, shard_params: bool = False) -> list[float]:
    from priml_b200.parallel.fused_fsdp import FusedFullySharded

    def strategy():  # noqa: ANN202
        return FusedFullySharded.Config(device="cpu", shard_params=shard_params)

    batches = _batches(4)

    def run(step, seqs):  # noqa: ANN001, ANN202
        out = []
        for seq in seqs:
            local = seq.chunk(world)[rank]
            o = step.train_step(tokens=local[:, :-1], targets=local[:, 1:])
            out.append(float(o["loss"].float().mean()))
        return out

    torch.manual_seed(0)
    a = _cfg(strategy()).make()
    straight = run(a, batches)
    torch.manual_seed(0)
    b = _cfg(strategy()).make()
    run(b, batches[:2])
    sd = {"model": b.model.state_dict(), "optimizer": b.optimizer.state_dict()}
    torch.manual_seed(123)
    c = _cfg(strategy()).make()
    c.model.load_state_dict(sd["model"])
    c.optimizer.load_state_dict(sd["optimizer"])
    resumed = run(c, batches[2:])
    return [straight[2] - resumed[0], straight[3] - resumed[1]]


@pytest.mark.parametrize("shard_params", [False, True])
def test_sharded_checkpoint_roundtrip_resumes_exactly(shard_params: bool) -> None:
    diffs = run_ranks(_resume, 2, shard_params, mesh_shape={"dp": 2})
    for d in diffs:
        assert all(abs(x) < 1e-6 for x in d), diffs


@pytest.mark.parametrize("accumulate", [1, 2])
def test_sharded_weights_match_resident_weights(accumulate: int) -> None:
    """Each rank keeping 1/R of the bf16 weights and gathering blocks into rotating windows
    computes exactly what resident weights compute."""
    resident = run_ranks(_sharded, 2, 4, accumulate, False, mesh_shape={"dp": 2})
    sharded = run_ranks(_sharded, 2, 4, accumulate, True, mesh_shape={"dp": 2})
    for r in range(2):
        assert sharded[r]["losses"] == resident[r]["losses"]
        assert sharded[r]["norms"] == resident[r]["norms"]
        for k, v in resident[r]["weights"].items():
            assert torch.equal(sharded[r]["weights"][k], v), k
        assert sharded[r]["shard_elems"] * 2 == sharded[r]["total_elems"]
