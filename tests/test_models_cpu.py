"""Model blocks on CPU: shapes, parameter layouts, and semantic equivalences."""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from priml_b200.models import (
    CausalLM,
    KVCache,
    MoE,
    MultiHeadLatentAttention,
    RMSNorm,
    RoPE,
    Router,
    SdpaFused,
    SdpaNaive,
    SelfAttention,
    SwiGLU,
    TransformerBlock,
    generate,
    window_mask,
)
from priml_b200.models.presets import tiny_lm
from priml_b200.ops import reference


def test_state_dict_names_match_reference_layout() -> None:
    m = CausalLM.Config(64, channels=32, num_layers=2, block=TransformerBlock.Config(
        attn=SelfAttention.Config(heads=4, num_heads_kv=2), ffn=SwiGLU.Config(channels_hidden=48))).make()  # fmt: skip
    sd = m.state_dict()
    assert sd["blocks.0.attn.proj_qkv.weight"].shape == (4 + 2 * 2, 8, 32)
    assert sd["blocks.1.ffn.up_proj.weight"].shape == (96, 32)
    assert sd["blocks.1.ffn.down_proj.weight"].shape == (32, 48)
    assert sd["embed.weight"].shape == (64, 32)
    assert sd["lm_head.weight"].shape == (64, 32)
    assert "final_norm.weight" not in sd  # no affine weight by default


def test_swiglu_gate_rows_first() -> None:
    torch.manual_seed(0)
    m = SwiGLU.Config(16, channels_hidden=8).make()
    x = torch.randn(3, 16)
    w = m.up_proj.weight
    ref = m.down_proj(F.silu(x @ w[:8].T) * (x @ w[8:].T))
    assert torch.allclose(m(x), ref, atol=1e-6)


def test_gqa_matches_expanded_heads() -> None:
    torch.manual_seed(0)
    q = torch.randn(2, 10, 4, 8)
    k = torch.randn(2, 10, 2, 8)
    v = torch.randn(2, 10, 2, 8)
    out = reference.attention(q, k, v, causal=True)
    kx, vx = k.repeat_interleave(2, dim=2), v.repeat_interleave(2, dim=2)
    sd = F.scaled_dot_product_attention(q.transpose(1, 2), kx.transpose(1, 2), vx.transpose(1, 2), is_causal=True)
    assert torch.allclose(out, sd.transpose(1, 2), atol=1e-5)
    assert torch.allclose(SdpaNaive()(q, k, v, is_causal=True), out, atol=1e-5)
    assert torch.allclose(SdpaFused()(q, k, v, is_causal=True), out, atol=1e-5)


def test_window_mask_admits_window_plus_self() -> None:
    q = torch.zeros(1, 6, 1, 4)
    m = window_mask(q, q, window=2)
    allowed = (m == 0).int()
    assert allowed[5].tolist() == [0, 0, 0, 1, 1, 1]
    out = reference.attention(torch.randn(1, 6, 1, 4), torch.randn(1, 6, 1, 4), torch.randn(1, 6, 1, 4), window=2)
    assert out.shape == (1, 6, 1, 4)


def test_rope_rotation_properties() -> None:
    rope = RoPE.Config(8, base=1e4).make()
    cos, sin = rope(torch.arange(5))
    assert cos.shape == (5, 1, 4)
    q = torch.randn(1, 5, 2, 8)
    k = torch.randn(1, 5, 2, 8)
    qr, kr = RoPE.rotate(q, k, cos, sin)
    assert torch.allclose(qr.norm(dim=-1), q.norm(dim=-1), atol=1e-5), "rotation preserves norms"
    # Relative-position property: <R(p)q, R(p)k> is position independent when q, k are shared.
    qq = q[:, :1].expand(1, 5, 2, 8)
    dots = (RoPE.rotate(qq, qq, cos, sin)[0] * RoPE.rotate(qq, qq, cos, sin)[1]).sum(-1)
    assert torch.allclose(dots, dots[:, :1].expand_as(dots), atol=1e-4)


def test_rmsnorm_eps_none_uses_dtype_eps() -> None:
    x = torch.randn(4, 16)
    m = RMSNorm.Config(16, eps=None).make()
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + torch.finfo(torch.float32).eps)
    assert torch.allclose(m(x), ref, atol=1e-6)


def test_kvcache_fifo_and_seen() -> None:
    c = KVCache.alloc(batch=1, heads=1, max_seq=4, channels_head=2)
    for i in range(6):
        k = torch.full((1, 1, 1, 2), float(i))
        c.update(k, k)
    assert c.length == 4 and c.seen == 6
    assert c.k[0, 0, :, 0].tolist() == [2.0, 3.0, 4.0, 5.0]


def test_kvcache_matches_naive_window_over_many_appends() -> None:
    """Mixed single- and multi-row appends far past capacity keep the newest rows in time order."""
    g = torch.Generator().manual_seed(3)
    for wrapped in (False, True):
        if wrapped:
            c = KVCache(torch.zeros(2, 3, 7, 4), torch.zeros(2, 3, 7, 5), length=0)
        else:
            c = KVCache.alloc(batch=2, heads=3, max_seq=7, channels_head=4, channels_v_head=5)
        hist_k, hist_v = [], []
        for step in range(40):
            s = int(torch.randint(1, 8, (1,), generator=g))
            k = torch.randn(2, 3, s, 4, generator=g)
            v = torch.randn(2, 3, s, 5, generator=g)
            hist_k.append(k)
            hist_v.append(v)
            kv, vv = c.update(k, v)
            want_k = torch.cat(hist_k, dim=-2)[..., -7:, :]
            want_v = torch.cat(hist_v, dim=-2)[..., -7:, :]
            assert torch.equal(kv, want_k) and torch.equal(vv, want_v), step
            assert c.length == want_k.shape[-2] and c.k.shape[-2] == 7
            assert torch.equal(c.k[..., : c.length, :], want_k)
        assert c.seen == sum(t.shape[-2] for t in hist_k)
        frozen = c.freeze()
        fk, _ = frozen.update(torch.ones(2, 3, 2, 4), torch.ones(2, 3, 2, 5))
        assert torch.equal(fk, want_k) and frozen.seen == c.seen


def test_generate_greedy_matches_full_forward() -> None:
    torch.manual_seed(0)
    m = tiny_lm().make().eval()
    prompt = torch.randint(0, 512, (2, 5))
    out = generate(m, prompt, max_new_tokens=4, temperature=0, max_seq_len=32)
    seq = prompt
    with torch.no_grad():
        for _ in range(4):
            nxt = m(seq)[:, -1].argmax(-1, keepdim=True)
            seq = torch.cat([seq, nxt], -1)
    assert torch.equal(out, seq)


def test_causal_lm_token_loss_equals_logits_ce() -> None:
    torch.manual_seed(0)
    m = tiny_lm().make()
    x = torch.randint(0, 512, (2, 9))
    loss = m.token_loss(x[:, :-1], x[:, 1:])
    ref = F.cross_entropy(m(x[:, :-1]).reshape(-1, 512), x[:, 1:].reshape(-1), reduction="none").reshape(2, 8)
    assert torch.allclose(loss, ref, atol=1e-5)


def test_mla_absorbed_equals_expanded() -> None:
    torch.manual_seed(0)
    mla = MultiHeadLatentAttention.Config(
        64, heads=4, channels_qk_nope_head=16, channels_qk_rope_head=8, channels_v_head=16, kv_lora_rank=32,
        rope=RoPE.Config(8, base=1e4),
    ).make()  # fmt: skip
    x = torch.randn(2, 12, 64)
    out, _ = mla(x)
    # Expanded evaluation order of the same weights.
    q = mla._project_q(x)
    q_nope, q_pe = q[..., :16], q[..., 16:]
    comp = mla.kv_a_proj(x)
    c_kv = mla.kv_a_layernorm(comp[..., :32])
    k_pe = comp[..., 32:].unsqueeze(-2)
    cos, sin = mla.rope(torch.arange(12))
    q_pe, k_pe = RoPE.rotate(q_pe, k_pe, cos, sin, interleave=True)
    exp = mla._expanded_attention(q_nope, q_pe, c_kv, k_pe.squeeze(-2))
    assert torch.allclose(out, mla.o_proj(exp), atol=1e-4)


def test_mla_decode_with_latent_cache_matches_prefill() -> None:
    torch.manual_seed(0)
    mla = MultiHeadLatentAttention.Config(32, heads=2, channels_qk_nope_head=8, channels_qk_rope_head=4,
                                          channels_v_head=8, kv_lora_rank=16, rope=RoPE.Config(4)).make().eval()  # fmt: skip
    x = torch.randn(1, 6, 32)
    full, _ = mla(x)
    cache = mla.alloc_kv_cache(batch=1, max_seq=8)
    outs = []
    for t in range(6):
        o, cache = mla(x[:, t : t + 1], cache=cache)
        outs.append(o)
    assert torch.allclose(torch.cat(outs, 1), full, atol=1e-4)


@pytest.mark.parametrize("scoring", ["softmax", "sigmoid"])
def test_moe_grouped_equals_per_expert_loop(scoring: str) -> None:
    torch.manual_seed(0)
    cfg = MoE.Config(16, router=Router.Config(num_experts=4, top_k=2, scoring_func=scoring),
                     expert=SwiGLU.Config(channels_hidden=8), num_shared_experts=1,
                     shared_expert=SwiGLU.Config(channels_hidden=8))  # fmt: skip
    moe = cfg.make()
    x = torch.randn(3, 5, 16)
    y = moe(x)
    xf = x.reshape(-1, 16)
    w, idx, _ = moe.router(xf)
    ref = torch.zeros_like(xf)
    for t in range(xf.shape[0]):
        for j in range(2):
            e = int(idx[t, j])
            g, u = (xf[t] @ moe.experts.up_proj[e].T).chunk(2)
            ref[t] += w[t, j] * (moe.experts.down_proj[e] @ (F.silu(g) * u))
    ref = ref + moe.shared_experts[0](xf)
    assert torch.allclose(y.reshape(-1, 16), ref, atol=1e-5)


def test_moe_state_dict_uses_per_expert_keys_and_roundtrips() -> None:
    torch.manual_seed(0)
    cfg = MoE.Config(8, router=Router.Config(num_experts=3, top_k=1), expert=SwiGLU.Config(channels_hidden=4))
    a = cfg.make()
    sd = a.state_dict()
    assert "experts.2.up_proj.weight" in sd and "experts.up_proj" not in sd
    b = cfg.make()
    b.load_state_dict(sd)
    assert torch.equal(a.experts.down_proj, b.experts.down_proj)


def test_moe_aux_loss_switch_formula() -> None:
    torch.manual_seed(0)
    moe = MoE.Config(8, router=Router.Config(num_experts=4, top_k=1), expert=SwiGLU.Config(channels_hidden=4),
                     aux_loss_weight=1.0).make()  # fmt: skip
    moe.train()
    moe(torch.randn(64, 8))
    assert moe.aux_loss > 0.0
    assert math.isfinite(float(moe.aux_loss))
