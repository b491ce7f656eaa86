"""Bit-for-bit goldens of model blocks at minimal width (CPU, host-agnostic numerics)."""

from __future__ import annotations

from pathlib import Path

import torch

from priml_b200.testing import assert_bfb_against_golden, host_agnostic_numerics, poison_free_pool

GOLDENS = Path(__file__).parent / "goldens"


def _block():  # noqa: ANN202
    from priml_b200.models.presets import dense_lm

    cfg = dense_lm(vocab=64, d_model=32, n_layers=1, n_heads=4, n_kv_heads=2, head_dim=8, ffn_hidden=64,
                   rope_theta=1e4)  # fmt: skip
    return cfg.make()


def _tokens():  # noqa: ANN202
    return torch.randint(0, 64, (2, 12), generator=torch.Generator().manual_seed(3))


def test_dense_lm_forward_golden() -> None:
    assert_bfb_against_golden(golden_dir=GOLDENS, golden_name="dense_lm_forward", build_module=_block,
                              build_input=_tokens, seed=0)  # fmt: skip


def _train_run(model, tokens):  # noqa: ANN001, ANN202
    from priml_b200.optimizers import FusedAdamW

    opt = FusedAdamW(model.parameters(), lr=1e-3, weight_decay=0.1)
    loss = model(tokens[:, :-1], targets=tokens[:, 1:]).mean()
    loss.backward()
    opt.step()
    return loss


def test_dense_lm_train_step_golden() -> None:
    assert_bfb_against_golden(golden_dir=GOLDENS, golden_name="dense_lm_train_step", build_module=_block,
                              build_input=_tokens, seed=1, run=_train_run)  # fmt: skip


def test_float64_mode_is_deterministic_and_keeps_float32() -> None:
    a = torch.randn(64, 64)
    with host_agnostic_numerics():
        x = (a @ a).sum(0).exp()
        y = a.clone()
        y.mul_(2.0).add_(1.0)
    assert x.dtype == torch.float32 and torch.equal(y, a * 2 + 1)
    ref = (a.double() @ a.double()).float().double().sum(0).float().double().exp().float()
    assert torch.equal(x, ref)
    poison_free_pool(blocks=4, device="cpu")
