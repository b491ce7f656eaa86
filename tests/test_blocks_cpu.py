"""Linear attention, value-gated attention and vision / mixer blocks on CPU."""

from __future__ import annotations

import torch

from priml_b200.models.attention import MultiStreamAttention
from priml_b200.models.gated_delta_net import GatedDeltaNet, gated_delta_chunked, gated_delta_recurrent
from priml_b200.models.rope import RoPE
from priml_b200.models.value_gated_attention import ValueGatedAttention
from priml_b200.models.vision import AdaLNZero, Conv2d, MLPMixerBlock, MMDiTBlock, Patchify, Unpatchify


def test_gated_delta_chunked_matches_recurrence() -> None:
    torch.manual_seed(0)
    B, S, H, dk, dv = 2, 37, 3, 8, 6
    q, k, v = torch.randn(B, S, H, dk), torch.randn(B, S, H, dk), torch.randn(B, S, H, dv)
    g = -torch.rand(B, S, H)
    beta = torch.rand(B, S, H)
    ref = gated_delta_recurrent(q, k, v, g, beta)
    for chunk in (8, 16, 64):
        got = gated_delta_chunked(q, k, v, g, beta, chunk=chunk)
        assert torch.allclose(got, ref, atol=1e-4), (chunk, float((got - ref).abs().max()))


def test_gated_delta_net_module_runs_and_backprops() -> None:
    torch.manual_seed(0)
    m = GatedDeltaNet.Config(32, heads_k=2, heads_v=4, channels_k_head=8, channels_v_head=8, chunk_size=8).make()
    x = torch.randn(2, 20, 32, requires_grad=True)
    y = m(x)
    assert y.shape == x.shape
    y.sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()


def test_value_gated_attention_zero_init_output() -> None:
    m = ValueGatedAttention.Config(64, channels_head=16, window=4).make()
    x = torch.randn(2, 10, 64)
    cos, sin = RoPE.Config(16).make()(torch.arange(10))
    out = m(x, cos_sin=(cos, sin), value_embedding=torch.randn(2, 10, 64))
    assert out.shape == x.shape
    assert float(out.detach().abs().max()) == 0.0, "proj_out is zero-initialized"


def test_patchify_roundtrip_and_vision_blocks() -> None:
    x = torch.randn(2, 3, 8, 6)
    p = Patchify.Config(3, patch_size=[2, 3]).make()
    tokens = p(x)
    assert tokens.shape == (2, 8, 18)
    back = Unpatchify.Config(3, patch_size=[2, 3]).make()(tokens, grid=[4, 2])
    assert torch.equal(back, x)
    conv = Conv2d.Config(3, 5).make()
    assert conv(x).shape == (2, 5, 8, 6)
    mix = MLPMixerBlock.Config(16, seq_len=10).make()
    assert mix(torch.randn(2, 10, 16)).shape == (2, 10, 16)
    blk = MMDiTBlock.Config(32, cond_dim=8, attn=MultiStreamAttention.Config(heads=4)).make()
    xs = [torch.randn(2, 5, 32), torch.randn(2, 3, 32)]
    out = blk(xs, c=torch.randn(2, 8))
    assert [o.shape for o in out] == [x.shape for x in xs]
    ada = AdaLNZero.Config(4, cond_dim=3).make()(torch.randn(2, 3))
    assert float(ada.attn_gate.abs().max()) == 0.0
