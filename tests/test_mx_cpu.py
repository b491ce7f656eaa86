"""MXFP8 quantization rule and the quantized training path (CPU reference kernels)."""

from __future__ import annotations

import pytest
import torch

from priml_b200.ops.mx import mx_dequantize_ref, mx_fake_quant, mx_linear, mx_quantize_ref


def test_scale_rule_follows_ocp_mx() -> None:
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 96, generator=g) * torch.logspace(-6, 6, 4).unsqueeze(1)
    x[0, :32] = 0.0  # an all-zero block
    x[1, 32:64] = 0.0
    x[1, 40] = 3.0  # amax 3: floor(log2 3) = 1 -> shared exponent 1 - 8
    q, e = mx_quantize_ref(x)
    assert int(e[0, 0]) == -127 and torch.all(q[0, :32].float() == 0)
    assert int(e[1, 1]) == 1 - 8
    assert float(q.float().abs().max()) <= 448.0
    # every block's largest magnitude lands in [256, 448] (no wasted range) unless the block is zero
    blocks = q.float().abs().view(4, 3, 32).amax(-1)
    assert torch.all((blocks == 0) | ((blocks >= 256) & (blocks <= 448)))
    # E4M3 keeps 3 mantissa bits: round-to-nearest error <= 2^-4 relative for values in the normal range
    # (scaled magnitudes above 448 saturate by the OCP rule: the block maximum lands in [256, 512))
    deq = mx_dequantize_ref(q, e)
    scaled = x.abs() / 2.0 ** e.repeat_interleave(32, 1).float()
    normal = (scaled >= 2**-6) & (scaled <= 448)
    rel = ((deq - x).abs() / x.abs().clamp_min(1e-30))[normal]
    assert float(rel.max()) <= 2**-4 + 1e-7
    sat = scaled > 464  # rounds past the largest finite E4M3 value
    assert torch.all(deq.abs()[sat] == 448 * 2.0 ** e.repeat_interleave(32, 1).float()[sat])


def test_fake_quant_along_either_dim() -> None:
    x = torch.randn(64, 96)
    a = mx_fake_quant(x, 0)
    b = mx_fake_quant(x.t().contiguous(), -1).t()
    assert torch.equal(a, b)


def test_mx_linear_reference_grads_track_bf16() -> None:
    g = torch.Generator().manual_seed(1)
    x = torch.randn(64, 128, generator=g, requires_grad=True)
    w = (torch.randn(96, 128, generator=g) / 128**0.5).requires_grad_()
    y = mx_linear(x, w)
    yr = x @ w.t()
    assert float((y - yr).norm() / yr.norm()) < 0.05
    gy = torch.randn_like(y)
    dx, dw = torch.autograd.grad(y, (x, w), gy)
    rx, rw = torch.autograd.grad(yr, (x, w), gy)
    assert float((dx - rx).norm() / rx.norm()) < 0.06
    assert float((dw - rw).norm() / rw.norm()) < 0.06


@pytest.mark.parametrize("recipe", ["mxfp8", "rowwise_gw_hp"])
def test_quantized_training_converts_linears_and_trains(recipe: str) -> None:
    from priml_b200.loss import TokenCrossEntropy
    from priml_b200.models.presets import tiny_lm
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.train import Float8ModelQuantization, TrainStep

    def make(quant):  # noqa: ANN001, ANN202
        torch.manual_seed(0)
        cfg = TrainStep.Config(model=tiny_lm(), optimizer=FusedAdamW.Config(lr=3e-3), loss=TokenCrossEntropy.Config(),
                               gradient_clip_norm=1.0)  # fmt: skip
        if quant is not None:
            cfg.model_quantization = quant
        return cfg.make()

    ref = make(None)
    mx = make(Float8ModelQuantization.Config(recipe=recipe))
    names = [n for n, m in mx.model.named_modules() if type(m).__name__.startswith("MXFP8")]
    assert names and all(n.rsplit(".", 1)[-1] in ("down_proj", "up_proj", "proj_out", "lm_head") for n in names), names
    assert sorted(mx.model.state_dict()) == sorted(ref.model.state_dict())
    seq = torch.randint(0, 512, (4, 65), generator=torch.Generator().manual_seed(2))
    losses = []
    for step in (ref, mx):
        out = [float(step.train_step(tokens=seq[:, :-1], targets=seq[:, 1:])["loss"].mean()) for _ in range(3)]
        losses.append(out)
    for a, b in zip(losses[1], losses[0], strict=True):
        assert abs(a - b) < 0.02 * abs(b), losses
    assert losses[1][-1] < losses[1][0]
