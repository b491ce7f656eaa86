"""Expert parallelism: device-side plan, exchange, expert sharding and gradients on gloo ranks.

The exchange runs the all-gather oracle communicator with the same plan,
row layout, autograd and gradient rules as the NVLink kernels.
"""

from __future__ import annotations

import torch

from priml_b200.testing import run_ranks


def _cfg(parallelism):  # noqa: ANN001, ANN202
    from priml_b200.loss import TokenCrossEntropy
    from priml_b200.models.presets import tiny_moe_lm
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.train import TrainStep

    return TrainStep.Config(
        model=tiny_moe_lm(),
        optimizer=FusedAdamW.Config(lr=3e-3, betas=(0.9, 0.95), weight_decay=0.1),
        loss=TokenCrossEntropy.Config(),
        parallelism=parallelism,
        gradient_clip_norm=1.0,
    )


def _batches(n: int) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 512, (8, 33), generator=g) for _ in range(n)]


def _ep(rank: int, world: int, steps: int) -> dict:
    from priml_b200.parallel.expert import ExpertParallel

    torch.manual_seed(0)
    step = _cfg(ExpertParallel.Config()).make()
    losses, norms = [], []
    for seq in _batches(steps):
        local = seq.chunk(world)[rank]
        out = step.train_step(tokens=local[:, :-1], targets=local[:, 1:])
        t = out["loss"].detach().float().mean()
        torch.distributed.all_reduce(t)
        losses.append(float(t) / world)
        norms.append(float(step.last_grad_norm))
    sd = step.model.state_dict()
    experts = sorted(k for k in sd if ".experts." in k)
    return {"losses": losses, "norms": norms, "experts": experts,
            "shape": tuple(step.model.blocks[0].ffn.experts.up_proj.shape)}  # fmt: skip


def _single(steps: int) -> dict:
    torch.manual_seed(0)
    step = _cfg(None).make()
    losses, norms = [], []
    for seq in _batches(steps):
        out = step.train_step(tokens=seq[:, :-1], targets=seq[:, 1:])
        losses.append(float(out["loss"].float().mean()))
        norms.append(float(step.last_grad_norm))
    return {"losses": losses, "norms": norms}


def _plan_body(rank: int, world: int) -> dict:
    from priml_b200.parallel.expert import ep_plan

    g = torch.Generator().manual_seed(rank)
    idx = torch.randint(0, 8, (10, 2), generator=g)
    plan = ep_plan(idx, 8, rank, world)
    return {"idx": idx, "dest_rank": plan.dest_rank, "dest_row": plan.dest_row, "seg": plan.seg_start,
            "tot": plan.totals, "cap": plan.cap}  # fmt: skip


def test_plan_lays_out_aligned_segments_in_rank_order() -> None:
    out = run_ranks(_plan_body, 2, mesh_shape={"dp": 2})
    for owner in range(2):
        seg = out[owner]["seg"].tolist()
        assert all(s % 128 == 0 for s in seg)
        rows = []
        for src in range(2):
            sel = out[src]["dest_rank"] == owner
            rows += out[src]["dest_row"][sel].tolist()
        # every slot routed to this owner lands on its own row, inside its expert's segment
        assert len(rows) == len(set(rows)) == int(out[owner]["tot"].sum())
        assert max(rows) < seg[-1] <= out[owner]["cap"]


def test_ep2_matches_single_process() -> None:
    ref = _single(3)
    two = run_ranks(_ep, 2, 3, mesh_shape={"dp": 2})
    assert two[0]["shape"][0] == 4  # 8 experts over 2 ranks
    # state dict keys name the global experts
    assert two[0]["experts"] != two[1]["experts"]
    assert "blocks.0.ffn.experts.7.up_proj.weight" in two[1]["experts"]
    for a, b in zip(two[0]["losses"], ref["losses"], strict=True):
        assert abs(a - b) < 2e-3 * max(1.0, abs(b)), (two[0]["losses"], ref["losses"])
    for a, b in zip(two[0]["norms"], ref["norms"], strict=True):
        assert abs(a - b) < 1e-2 * max(1.0, abs(b)), (two[0]["norms"], ref["norms"])


def _routes_body(rank: int, world: int) -> dict:
    from priml_b200.parallel.expert import ep_plan, ep_routes

    g = torch.Generator().manual_seed(rank)
    idx = torch.randint(0, 8, (10, 3), generator=g)
    plan = ep_plan(idx, 8, rank, world)
    routes = ep_routes(idx, 8, rank, world)
    return {"dest_rank": plan.dest_rank, "dest_row": plan.dest_row, "seg": plan.seg_start, "cap": plan.cap,
            "origin": routes.origin, "row_src": routes.row_src, "rseg": routes.seg_start, "rcap": routes.cap}  # fmt: skip


def test_routes_name_the_source_of_every_row_the_plan_sends() -> None:
    """The owner-side routes of the fused exchange agree with the source-side plan."""
    out = run_ranks(_routes_body, 2, mesh_shape={"dp": 2})
    for owner in range(2):
        o = out[owner]
        assert torch.equal(o["rseg"], o["seg"]) and o["rcap"] == o["cap"]
        expect = torch.full_like(o["origin"], -1)
        expect_src = torch.full_like(o["row_src"], -1)
        for src in range(2):
            sel = torch.nonzero(out[src]["dest_rank"] == owner).flatten()
            rows = out[src]["dest_row"][sel]
            expect[rows] = ((src << 24) | sel).to(torch.int32)
            expect_src[rows] = ((src << 24) | (sel // 3)).to(torch.int32)
        assert torch.equal(o["origin"], expect)
        assert torch.equal(o["row_src"], expect_src)
