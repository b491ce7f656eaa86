"""tcgen05 flash attention vs an fp32 PyTorch reference of the same op."""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, causal, scale, window):
    from priml_b200.ops import reference

    return reference.attention(q.float(), k.float(), v.float(), causal=causal, scale=scale, window=window)


def _err(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


CASES = [
    # B, S, T, H, Hkv, D, causal, window
    (2, 256, 256, 4, 2, 64, True, None),
    (1, 300, 300, 4, 1, 64, True, None),
    (2, 384, 384, 2, 2, 128, True, None),
    (1, 256, 256, 4, 4, 64, False, None),
    (1, 512, 512, 2, 1, 64, True, 100),
    (1, 128, 384, 2, 2, 64, True, None),
    (3, 81, 81, 8, 8, 64, False, None),  # sequence length not a multiple of 4 (padded delta rows)
    (1, 917, 917, 2, 2, 64, False, None),
]


@pytest.mark.parametrize("B,S,T,H,Hkv,D,causal,window", CASES)
def test_flash_attention_fwd_bwd(B, S, T, H, Hkv, D, causal, window) -> None:
    from priml_b200.ops import native
    from priml_b200.ops.attention_fn import FlashAttnFn

    torch.manual_seed(0)
    q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    scale = 1.0 / math.sqrt(D)
    o = FlashAttnFn.apply(q, k, v, causal, scale, -1 if window is None else window)
    do = torch.randn_like(o)
    o.backward(do)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    orf = _ref(qr, kr, vr, causal, scale, window)
    orf.backward(do.float())
    torch.cuda.synchronize()
    assert native().read_status(True) == 0
    assert _err(o, orf) < 2e-2
    assert _err(q.grad, qr.grad) < 3e-2
    assert _err(k.grad, kr.grad) < 3e-2
    assert _err(v.grad, vr.grad) < 3e-2


def test_flash_attention_strided_v() -> None:
    """V as a strided view of a fused QKV buffer (the layout SelfAttention produces)."""
    from priml_b200.ops.attention_fn import FlashAttnFn

    torch.manual_seed(1)
    B, S, H, Hkv, D = 2, 256, 4, 2, 64
    qkv = torch.randn(B, S, H + 2 * Hkv, D, device="cuda", dtype=torch.bfloat16)
    q, k, v = qkv.split([H, Hkv, Hkv], dim=2)
    q, k = q.contiguous(), k.contiguous()
    o = FlashAttnFn.apply(q, k, v, True, 1 / 8, -1)
    assert _err(o, _ref(q, k, v, True, 1 / 8, None)) < 2e-2


@pytest.mark.parametrize("D,window", [(128, 256), (64, 256), (128, None), (64, 100)])
def test_flash_attention_rows_rescale_independently(D: int, window) -> None:  # noqa: ANN001
    """RMS-normalized q / k give scores of magnitude ~sqrt(D), so rows of one warp move their
    running max at different tiles (windows make their first visible tile differ too)."""
    from priml_b200.ops import native
    from priml_b200.ops.attention_fn import FlashAttnFn

    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, v = (torch.randn(4, 512, 4, D, device="cuda", generator=g) for _ in range(3))
    q = (q / q.pow(2).mean(-1, keepdim=True).sqrt()).to(torch.bfloat16).requires_grad_()
    k = (k / k.pow(2).mean(-1, keepdim=True).sqrt()).to(torch.bfloat16).requires_grad_()
    v = v.to(torch.bfloat16).requires_grad_()
    scale = D**-0.5
    o = FlashAttnFn.apply(q, k, v, True, scale, -1 if window is None else window)
    go = torch.randn_like(o)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), go)
    qf, kf, vf = (x.detach().float().requires_grad_() for x in (q, k, v))
    idx = torch.arange(512, device="cuda")
    off = idx[:, None] - idx[None, :]
    mask = (off >= 0) & ((off <= window) if window is not None else True)
    ref = torch.nn.functional.scaled_dot_product_attention(qf.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2),
                                                           attn_mask=mask, scale=scale).transpose(1, 2)  # fmt: skip
    rq, rk, rv = torch.autograd.grad(ref, (qf, kf, vf), go.float())
    assert _err(o, ref) < 2e-2
    assert _err(dq, rq) < 5e-2 and _err(dk, rk) < 5e-2 and _err(dv, rv) < 5e-2
    assert int(native().read_status(True)) == 0


MLA_CASES = [
    # B, S, T, H, Hkv, causal, window -- query/key head dim 192 (128 + 64 rotary), value head dim 128
    (1, 256, 256, 4, 4, True, None),
    (2, 300, 300, 2, 2, True, None),
    (1, 256, 256, 2, 2, False, None),
    (1, 128, 384, 2, 2, True, None),
    (1, 384, 384, 2, 1, True, 100),
]


@pytest.mark.parametrize("B,S,T,H,Hkv,causal,window", MLA_CASES)
def test_latent_attention_head_dims_fwd_bwd(B, S, T, H, Hkv, causal, window) -> None:  # noqa: ANN001
    """Multi-head latent attention shapes: q / k 192 wide, v 128 wide, against the fp32 oracle."""
    from priml_b200.ops import native
    from priml_b200.ops.attention_fn import FlashAttnFn

    torch.manual_seed(2)
    q = torch.randn(B, S, H, 192, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, T, Hkv, 192, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, T, Hkv, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    scale = 1.0 / math.sqrt(192)
    o = FlashAttnFn.apply(q, k, v, causal, scale, -1 if window is None else window)
    assert o.shape == (B, S, H, 128)
    do = torch.randn_like(o)
    o.backward(do)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    orf = _ref(qr, kr, vr, causal, scale, window)
    orf.backward(do.float())
    torch.cuda.synchronize()
    assert native().read_status(True) == 0
    assert _err(o, orf) < 2e-2
    assert _err(q.grad, qr.grad) < 3e-2
    assert _err(k.grad, kr.grad) < 3e-2
    assert _err(v.grad, vr.grad) < 3e-2


def test_mla_module_training_path_uses_the_kernel() -> None:
    """The MLA block's expanded training attention matches the absorbed oracle path."""
    from priml_b200.models.mla import MultiHeadLatentAttention
    from priml_b200.models.rope import RoPE

    torch.manual_seed(0)
    mla = MultiHeadLatentAttention.Config(channels_in=256, heads=4, kv_lora_rank=64, channels_qk_nope_head=128,
                                          channels_qk_rope_head=64, channels_v_head=128,
                                          rope=RoPE.Config(64, base=1e4)).make().cuda().train()  # fmt: skip
    x = torch.randn(2, 256, 256, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        fast, _ = mla(x)
        mla.eval()
        slow, _ = mla(x)  # the absorbed path (einsums), not the kernel
    assert _err(fast, slow) < 3e-2
