"""Latent-space MLA decode kernel (``ops/csrc/mla_decode.cu``) against an fp32 PyTorch oracle.

Covers one to many key tiles, splits of the key axis merged by the combine kernel,
partial head groups (H not a multiple of the 16- or 32-head tile), per-sequence
lengths (including an empty sequence), caches that are strided slices of a larger
buffer, and the MLA module's one-token decode step against its einsum order.
"""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _err(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


@pytest.mark.parametrize(
    "B,H,T,use_len",
    [(1, 16, 1, False), (3, 16, 100, False), (2, 16, 700, True), (4, 16, 4096, False), (2, 20, 333, True),
     (1, 64, 2048, False), (2, 32, 129, True), (64, 16, 1024, True)],  # fmt: skip
)
def test_mla_decode_matches_fp32_oracle(B, H, T, use_len) -> None:  # noqa: ANN001
    from priml_b200 import ops
    from priml_b200.ops import native, reference

    torch.manual_seed(0)
    dev = "cuda"
    # caches are slices of longer buffers, so the sequence stride is not T * width
    c_buf = torch.randn(B, T + 37, 512, device=dev).to(torch.bfloat16)
    r_buf = torch.randn(B, T + 37, 64, device=dev).to(torch.bfloat16)
    c_kv, k_pe = c_buf[:, :T], r_buf[:, :T]
    q = (torch.randn(B, H, 576, device=dev) * 0.5).to(torch.bfloat16)
    lengths = None
    if use_len:
        lengths = torch.randint(1, T + 1, (B,), device=dev, dtype=torch.int32)
        lengths[0] = 0 if B > 1 else lengths[0]  # an empty sequence gives zeros
    scale = 1.0 / math.sqrt(192)
    for _ in range(2):
        got = ops.mla_decode(q, c_kv, k_pe, scale=scale, lengths=lengths)
        torch.cuda.synchronize()
        assert int(native().read_status(True)) == 0
        ref = reference.mla_decode(q.float(), c_kv.float(), k_pe.float(), scale=scale, lengths=lengths)
        assert torch.isfinite(got.float()).all()
        assert _err(got, ref) < 2e-2, _err(got, ref)
        if use_len and B > 1:
            assert float(got[0].float().abs().max()) == 0.0


def test_mla_module_decode_step_uses_kernel_and_matches_einsum_order(monkeypatch) -> None:  # noqa: ANN001
    from priml_b200.models.mla import MultiHeadLatentAttention

    torch.manual_seed(0)
    mla = MultiHeadLatentAttention.Config(channels_in=512, heads=16, kv_lora_rank=512, channels_qk_nope_head=128,
                                          channels_qk_rope_head=64, channels_v_head=128).make()  # fmt: skip
    mla = mla.cuda().to(torch.bfloat16).eval()
    x = torch.randn(3, 300, 512, device="cuda").to(torch.bfloat16)
    step = torch.randn(3, 1, 512, device="cuda").to(torch.bfloat16)
    calls = []
    real = MultiHeadLatentAttention._latent_decode_kernel

    def spy(self, *a):  # noqa: ANN001, ANN202
        used = real(self, *a)
        calls.append(used)
        return used

    with torch.no_grad():
        _, cache = mla(x)
        monkeypatch.setattr(MultiHeadLatentAttention, "_latent_decode_kernel", spy)
        y_kernel, _ = mla(step, cache=cache.clone() if hasattr(cache, "clone") else cache)
        assert calls and calls[-1], "the decode step did not take the kernel"
        monkeypatch.setattr(MultiHeadLatentAttention, "_latent_decode_kernel", lambda self, *a: False)
        _, cache2 = mla(x)
        y_einsum, _ = mla(step, cache=cache2)
    assert _err(y_kernel, y_einsum) < 3e-2, _err(y_kernel, y_einsum)
