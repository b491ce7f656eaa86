"""Optimizers, schedules, TrainStep / TrainLoop, checkpointing and EMA on CPU."""

from __future__ import annotations

import math
import os

import pytest
import torch

from priml_b200.config import PartialConfig
from priml_b200.data import SyntheticTokens
from priml_b200.loss import TokenCrossEntropy
from priml_b200.math import schedules
from priml_b200.models.presets import tiny_lm
from priml_b200.ops import reference
from priml_b200.optimizers import (
    AdamATan2,
    CompositeOptimizer,
    FusedAdamW,
    Muon,
    NorMuon,
    SignSGD,
    complement,
    excluding,
    matching,
)
from priml_b200.train import EMA, Checkpointer, TrainLoop, TrainStep


def test_fused_adamw_matches_formula() -> None:
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(10))
    ref = p.detach().clone()
    m, v = torch.zeros(10), torch.zeros(10)
    opt = FusedAdamW([p], lr=0.1, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(1, 4):
        g = torch.randn(10)
        p.grad = g.clone()
        opt.step()
        reference.adamw_([ref], [g], [m], [v], step=step, lr=0.1, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
    assert torch.allclose(p.detach(), ref, atol=1e-6)
    st = opt.state[p]
    assert set(st) == {"step", "first_moment", "second_moment"}


def test_fused_adamw_matches_torch_adamw_closely() -> None:
    torch.manual_seed(0)
    a = torch.nn.Parameter(torch.randn(5, 5))
    b = torch.nn.Parameter(a.detach().clone())
    oa = FusedAdamW([a], lr=1e-2, betas=(0.9, 0.99), weight_decay=0.05)
    ob = torch.optim.AdamW([b], lr=1e-2, betas=(0.9, 0.99), weight_decay=0.05)
    for _ in range(5):
        g = torch.randn(5, 5)
        a.grad, b.grad = g.clone(), g.clone()
        oa.step()
        ob.step()
    assert torch.allclose(a, b, atol=1e-5)


def test_muon_orthogonalizes_update() -> None:
    torch.manual_seed(0)
    w = torch.nn.Parameter(torch.zeros(16, 32))
    opt = Muon([w], lr=1.0, weight_decay=None, nesterov=False, momentum=0.0)
    w.grad = torch.randn(16, 32)
    opt.step()
    upd = -w.detach() / math.sqrt(max(1, 16 / 32))
    s = torch.linalg.svdvals(upd.float())
    assert float(s.max()) < 1.5 and float(s.min()) > 0.3


def test_normuon_and_others_step() -> None:
    torch.manual_seed(0)
    ws = [torch.nn.Parameter(torch.randn(8, 4)) for _ in range(3)]
    for w in ws:
        w.grad = torch.randn_like(w)
    before = [w.detach().clone() for w in ws]
    NorMuon(ws, lr=0.01).step()
    assert all(not torch.equal(a, b) for a, b in zip(before, ws, strict=True))
    p = torch.nn.Parameter(torch.randn(6))
    p.grad = torch.randn(6)
    AdamATan2([p]).step()
    q = torch.nn.Parameter(torch.zeros(4, 3))
    q.grad = torch.tensor([[1.0, -2, 0], [0, 0, 0], [3, 0, 0], [0, 0, 0]])
    SignSGD([q], lr=0.5, weight_decay=0.0, aggregate_distributed=False).step()
    assert q.detach()[0].tolist() == [-0.5, 0.5, 0.0]


def test_composite_routes_by_selector() -> None:
    m = tiny_lm().make()
    cfg = CompositeOptimizer.Config(
        optimizers=[Muon.Config(lr=0.01), FusedAdamW.Config(lr=1e-3)],
        select=[excluding(Muon.eligible_tensor, "embed", "lm_head"), complement(excluding(Muon.eligible_tensor, "embed", "lm_head"))],
    )  # fmt: skip
    opt = cfg.make()(m)
    names = {id(p): n for n, p in m.named_parameters()}
    muon_names = {names[id(p)] for g in opt.optimizers[0].param_groups for p in g["params"]}
    assert all("embed" not in n and "lm_head" not in n for n in muon_names)
    assert matching("embed")("embed.weight", None)  # type: ignore[arg-type]
    sd = opt.state_dict()
    assert len(sd["optimizers"]) == 2


def test_schedules() -> None:
    assert schedules.cosine(0.0) == 1.0 and abs(schedules.cosine(1.0)) < 1e-12
    assert schedules.trapezoidal(0.25, flat=0.5) == 1.0
    assert abs(schedules.trapezoidal(0.75, flat=0.5) - 0.5) < 1e-12
    assert schedules.warmup(0.05, fraction=0.1) == 0.5
    assert schedules.staircase(0.99, drops=3, gamma=0.1) == pytest.approx(1e-3)


def _loop_cfg(tmp: str, steps: int, save_every: int = 10) -> TrainLoop.Config:
    return TrainLoop.Config(
        step=TrainStep.Config(
            model=tiny_lm(),
            optimizer=FusedAdamW.Config(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1),
            loss=TokenCrossEntropy.Config(),
            learning_rate_scheduler=PartialConfig(schedules.constant),
        ),
        dataset=SyntheticTokens.Config(vocab_size=512, batch_size=8, seq_len=64, steps_per_epoch=10_000, pin_memory=False),
        max_steps=steps,
        num_steps_log=5,
        num_steps_eval=1_000_000,
        seed=0,
        working_dir=tmp,
        checkpointing=Checkpointer.Config(working_dir=os.path.join(tmp, "ckpt"), save_every=save_every),
    )


def test_tiny_lm_trains_20_steps_fp32_cpu(tmp_path) -> None:  # noqa: ANN001
    """The tiny decoder (vocab 512, d 128, 2 layers) takes 20 AdamW steps on CPU."""
    loop = _loop_cfg(str(tmp_path), 20).make()
    losses = []
    orig = loop.step.train_step

    def record(**batch):  # noqa: ANN003, ANN202
        out = orig(**batch)
        losses.append(float(out["loss"].float().mean()))
        return out

    loop.step.train_step = record  # type: ignore[method-assign]
    loop.run()
    assert len(losses) == 20
    assert all(math.isfinite(x) for x in losses)
    assert abs(losses[0] - math.log(512)) < 0.5
    assert sorted(os.listdir(tmp_path / "ckpt")) == ["step_00000010.pt", "step_00000020.pt"]


def test_resume_continues_from_checkpoint(tmp_path) -> None:  # noqa: ANN001
    _loop_cfg(str(tmp_path), 10, save_every=5).make().run()
    loop = _loop_cfg(str(tmp_path), 12, save_every=5).make()
    assert loop.global_step == 10
    loop.run()
    assert loop.global_step == 12


def test_overwrite_guard_refuses_shorter_run(tmp_path) -> None:  # noqa: ANN001
    _loop_cfg(str(tmp_path), 10, save_every=5).make().run()
    cfg = _loop_cfg(str(tmp_path), 10, save_every=5)
    cfg.checkpointing.resume = False
    with pytest.raises(RuntimeError, match="overwrite"):
        cfg.make()


def test_corrupt_latest_checkpoint_falls_back(tmp_path) -> None:  # noqa: ANN001
    _loop_cfg(str(tmp_path), 10, save_every=5).make().run()
    (tmp_path / "ckpt" / "step_00000010.pt").write_bytes(b"corrupt")
    loop = _loop_cfg(str(tmp_path), 12, save_every=5).make()
    assert loop.global_step == 5


def test_ema_param_dict_tracks_weights() -> None:
    """The reference's update rule: the shadow is taken at the first call, averaged from then on."""
    m = torch.nn.Linear(3, 3)
    ema = EMA.Config(decay=0.5, shadow_kind="param_dict").make()
    ema(m)  # shadow = current weights (averaging them with themselves)
    start = m.weight.detach().clone()
    with torch.no_grad():
        m.weight.add_(1.0)
    ema(m)
    with ema.apply_to(m):
        inside = m.weight.detach().clone()
    torch.testing.assert_close(inside, start + 0.5)
    torch.testing.assert_close(m.weight.detach(), start + 1.0)  # live weights come back
    state = ema.state_dict()
    assert set(state) == {"shadow_params", "shadow_buffers", "global_step", "local_step"}
    assert state["global_step"] == 2 and state["local_step"] == 2


def test_ema_warmup_seed_and_karras_schedule() -> None:
    from priml_b200.train.ema import karras_decay

    m = torch.nn.Linear(2, 2)
    ema = EMA.Config(decay=0.999, update_after_step=2, warmup_seed=True, decay_schedule=karras_decay).make()
    for i in range(2):
        with torch.no_grad():
            m.weight.fill_(float(i))
        ema(m)  # warmup calls only count
    assert ema.local_step == 0 and ema.global_step == 2
    with torch.no_grad():
        m.weight.fill_(10.0)
    ema(m)  # boundary: seeded from the live weights
    with torch.no_grad():
        m.weight.fill_(20.0)
    ema(m)  # first average: decay min(0.999, 2 / 11)
    d = 2 / 11
    with ema.apply_to(m):
        torch.testing.assert_close(m.weight.detach(), torch.full((2, 2), d * 10.0 + (1 - d) * 20.0))
    # module shadows checkpoint as a state dict and load before the first call
    mod = EMA.Config(decay=0.9).make()
    mod(m)
    fresh = EMA.Config(decay=0.9).make()
    fresh.load_state_dict(mod.state_dict())
    fresh(m)
    assert fresh.global_step == 2 and fresh.shadow_model is not None
