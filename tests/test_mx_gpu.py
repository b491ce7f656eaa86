"""MXFP8 kernels: quantizers (bit-exact vs the PyTorch reference) and the block-scaled tcgen05 GEMM."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _n():  # noqa: ANN202
    from priml_b200.ops import native

    return native()


def _unblock(sf: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """Blocked scale bytes -> int [rows, k / 32] (E8M0 bytes)."""
    nkg = (k + 127) // 128
    r = torch.arange(rows, device=sf.device).unsqueeze(1)
    kb = torch.arange(k // 32, device=sf.device).unsqueeze(0)
    off = ((r >> 7) * nkg + (kb >> 2)) * 512 + 16 * (r & 31) + 4 * ((r & 127) >> 5) + (kb & 3)
    return sf.long()[off]


@pytest.mark.parametrize("rows,k", [(256, 256), (300, 96), (64, 1024)])
def test_quantize_matches_reference_bits(rows: int, k: int) -> None:
    from priml_b200.ops.mx import mx_quantize_ref

    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(rows, k, device="cuda", generator=g) * torch.logspace(-8, 8, k, device="cuda")).to(torch.bfloat16)
    x[:, :32] = 0
    q, sf = _n().mx_quantize(x, False)
    rq, re = mx_quantize_ref(x)
    assert torch.equal(q, rq.view(torch.uint8))
    assert torch.equal(_unblock(sf, rows, k), re.long() + 127)
    if rows % 32 == 0:
        qt, sft = _n().mx_quantize(x, True)
        tq, te = mx_quantize_ref(x.t().contiguous())
        assert torch.equal(qt, tq.view(torch.uint8))
        assert torch.equal(_unblock(sft, k, rows), te.long() + 127)


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (300, 520, 256), (1024, 768, 96), (2048, 2048, 1024)])
def test_mx_gemm_matches_dequantized_matmul(m: int, n: int, k: int) -> None:
    from priml_b200.ops import native
    from priml_b200.ops.mx import mx_dequantize_ref, mx_quantize_ref

    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, device="cuda", generator=g) * 3).to(torch.bfloat16)
    qa, sa = native().mx_quantize(a, False)
    qb, sb = native().mx_quantize(b, False)
    ref = mx_dequantize_ref(*mx_quantize_ref(a)) @ mx_dequantize_ref(*mx_quantize_ref(b)).t()
    out = torch.empty(m, n, device="cuda", dtype=torch.float32)
    native().mx_gemm(qa, sa, qb, sb, out, 1)
    torch.cuda.synchronize()
    assert float((out - ref).abs().max() / ref.abs().max()) < 1e-4
    out16 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    native().mx_gemm(qa, sa, qb, sb, out16, 0)
    assert float((out16.float() - ref).abs().max() / ref.abs().max()) < 1e-2
    native().mx_gemm(qa, sa, qb, sb, out, 2)  # accumulate: 2 x
    assert float((out - 2 * ref).abs().max() / ref.abs().max()) < 2e-4
    assert int(native().read_status(True)) == 0


@pytest.mark.parametrize("wgrad_hp", [False, True])
def test_mx_linear_matches_reference_path(wgrad_hp: bool) -> None:
    from priml_b200.ops.mx import _MXLinearRef, mx_linear

    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(512, 384, device="cuda", generator=g).to(torch.bfloat16).requires_grad_()
    w = (torch.randn(640, 384, device="cuda", generator=g) / 384**0.5).requires_grad_()
    y = mx_linear(x, w, wgrad_high_precision=wgrad_hp)
    gy = torch.randn(512, 640, device="cuda", generator=g).to(torch.bfloat16)
    dx, dw = torch.autograd.grad(y, (x, w), gy)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().to(torch.bfloat16).float().requires_grad_()
    yr = _MXLinearRef.apply(xr, wr, wgrad_hp)
    rx, rw = torch.autograd.grad(yr, (xr, wr), gy.float())

    def rel(a: torch.Tensor, b: torch.Tensor) -> float:
        return float((a.float() - b).abs().max() / b.abs().max())

    assert rel(y.detach(), yr.detach()) < 1e-2
    assert rel(dx, rx) < 1e-2
    assert rel(dw, rw) < 1e-2


def test_mx_weight_copies_follow_optimizer_steps() -> None:
    """The fused AdamW kernel rewrites the weights in place; the cached MXFP8 weight copies must
    not outlive that: after a step the quantized forward equals a fresh quantization of the new
    weights."""
    from priml_b200.ops.mx import _MXLinearRef, mx_linear
    from priml_b200.optimizers import FusedAdamW

    g = torch.Generator(device="cuda").manual_seed(3)
    w = torch.nn.Parameter(torch.randn(256, 128, device="cuda", generator=g) / 128**0.5)
    x = torch.randn(64, 128, device="cuda", generator=g).to(torch.bfloat16)
    opt = FusedAdamW([w], lr=0.05)
    for _ in range(3):
        y = mx_linear(x, w)
        y.float().square().mean().backward()
        opt.step()
        opt.zero_grad()
    fresh = _MXLinearRef.apply(x.float(), w.detach().to(torch.bfloat16).float(), False)
    y = mx_linear(x, w).detach().float()
    assert float((y - fresh).abs().max() / fresh.abs().max()) < 1e-2


def test_mxfp8_loss_curve_tracks_bf16() -> None:
    """The first 40 steps of the same run with MXFP8 linear layers stay on the bf16 curve."""
    from priml_b200.train.precision_curve import run_curve

    # lr 5e-4 keeps both runs out of the loss-spike regime (at 2e-3 a spike near step 10 sends
    # bf16 and either MXFP8 GEMM onto different chaotic paths), so the gap measures precision
    kw = {"layers": 2, "steps": 40, "seq": 256, "batch": 4, "d_model": 512, "heads": 8, "kv_heads": 4,
          "head_dim": 64, "ffn": 1536, "vocab": 4096, "lr": 5e-4}  # fmt: skip
    bf16 = run_curve(mxfp8=False, **kw)
    mx = run_curve(mxfp8=True, **kw)
    assert bf16[-1] < bf16[0] - 1.0 and mx[-1] < mx[0] - 1.0  # both learn
    gaps = [abs(a - b) for a, b in zip(bf16, mx, strict=True)]
    assert max(gaps[:5]) < 0.05, gaps[:5]
    assert sum(gaps[-10:]) / 10 < 0.15, (bf16[-10:], mx[-10:])
