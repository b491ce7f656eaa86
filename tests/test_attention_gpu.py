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
