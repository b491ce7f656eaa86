"""Losses against the reference's own implementations, same inputs and seeds.

DiffusionLoss (rectified flow, with and without Min-SNR weighting), the PPO
terms, categorical entropy with masked actions, the GAN generator loss, and the
RoPE-Mixed tables.
"""

from __future__ import annotations

import pytest
import torch

from priml_b200.testing.reference import load_reference, reference_available

pytestmark = pytest.mark.skipif(not reference_available(), reason="the reference copy is not present")


def _denoiser(x: torch.Tensor, sigma: torch.Tensor) -> torch.Tensor:
    return 0.5 * x - 0.1 * sigma


@pytest.mark.parametrize("snr_gamma", [0.0, 5.0])
def test_diffusion_loss_matches_reference(snr_gamma: float) -> None:
    load_reference()
    from priml.loss.diffusion import DiffusionLoss as Ref

    from priml_b200.loss import DiffusionLoss

    x0 = torch.randn(6, 3, 4, 4, generator=torch.Generator().manual_seed(0))
    torch.manual_seed(1)
    ref = Ref.Config(snr_gamma=snr_gamma).make()(denoiser=_denoiser, x0=x0)
    torch.manual_seed(1)
    ours = DiffusionLoss.Config(snr_gamma=snr_gamma).make()(denoiser=_denoiser, x0=x0)
    for key in ("loss", "x_denoised", "eps_denoised", "log_snr", "log_sigma"):
        torch.testing.assert_close(ours[key], ref[key], rtol=1e-5, atol=1e-6, msg=key)
    assert ours["loss"].shape == (6,)


def test_ppo_terms_and_entropy_match_reference() -> None:
    load_reference()
    from priml.loss.policy_gradient import categorical_entropy as ref_entropy
    from priml.loss.policy_gradient import clipped_policy_loss as ref_ppo

    from priml_b200.loss import categorical_entropy, clipped_policy_loss

    g = torch.Generator().manual_seed(2)
    kw = {name: torch.randn(64, generator=g) for name in
          ("log_probs", "behavior_log_probs", "advantages", "values", "behavior_values", "targets", "entropy")}  # fmt: skip
    kw["log_probs"] = kw["behavior_log_probs"] + 0.3 * kw["log_probs"]
    for a, b in zip(clipped_policy_loss(**kw, clip_epsilon=0.2), ref_ppo(**kw, clip_epsilon=0.2), strict=True):
        torch.testing.assert_close(a, b)
    logits = torch.randn(5, 7, generator=g)
    logits[1, 3] = float("-inf")
    logp = logits.log_softmax(-1)
    torch.testing.assert_close(categorical_entropy(logp), ref_entropy(logp))
    assert torch.isfinite(categorical_entropy(logp)).all()


def test_adversarial_loss_matches_reference() -> None:
    load_reference()
    from priml.loss.gan import AdversarialLoss as Ref

    from priml_b200.loss import AdversarialLoss

    g = torch.Generator().manual_seed(3)
    kw = {"fake_logits": torch.randn(4, 1, generator=g), "fake_media": torch.randn(4, 3, 8, generator=g),
          "real_media": torch.randn(4, 3, 8, generator=g)}  # fmt: skip
    cfg = {"adversarial_weight": 0.7, "content_weight": 3.0}
    torch.testing.assert_close(AdversarialLoss.Config(**cfg).make()(None, **kw)["loss"],
                               Ref.Config(**cfg).make()(None, **kw)["loss"])  # fmt: skip


@pytest.mark.parametrize("mode,learnable", [("cat", False), ("sum", True)])
def test_rope_mixed_tables_match_reference(mode: str, learnable: bool) -> None:
    load_reference()
    from priml.model.rope import RoPEMixed as Ref

    from priml_b200.models.rope import RoPEMixed

    dims = (16, 16)
    torch.manual_seed(4)
    ref = Ref.Config(dims, heads=4, base=100.0, reduction_mode=mode, learnable=learnable).make()
    torch.manual_seed(4)
    ours = RoPEMixed.Config(dims, heads=4, base=100.0, reduction_mode=mode, learnable=learnable).make()
    pos = torch.stack(torch.meshgrid(torch.arange(5), torch.arange(3), indexing="ij"), -1).reshape(-1, 2)
    for a, b in zip(ours(pos), ref(pos), strict=True):
        torch.testing.assert_close(a.float(), b.float(), rtol=1e-6, atol=1e-6)
    assert [p.requires_grad for p in ours.parameters()] == [p.requires_grad for p in ref.parameters()]
