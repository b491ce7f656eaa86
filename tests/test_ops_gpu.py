"""Numerics of the sm_100a kernels against fp32 PyTorch references of the same op."""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _native():
    from priml_b200.ops import native

    return native()


def _rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a.detach() - b.detach()).abs().max() / b.detach().abs().max().clamp_min(1e-6))


LAYOUTS = [(False, False), (False, True), (True, False), (True, True)]
SHAPES = [(128, 256, 64), (300, 520, 200), (1024, 2048, 512), (2048, 768, 1088), (300, 260, 96), (264, 512, 8200)]


@pytest.mark.parametrize("a_mn,b_mn", LAYOUTS)
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_layouts(a_mn: bool, b_mn: bool, m: int, n: int, k: int) -> None:
    from priml_b200.ops.functional import gemm

    if (a_mn and m % 8) or (b_mn and n % 8):
        pytest.skip("an M/N-major operand needs its contiguous extent to be a multiple of 8 (16-byte TMA rows)")
    torch.manual_seed(0)
    a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
    ref = a.float() @ b.float().T
    a_in = a.T.contiguous() if a_mn else a
    b_in = b.T.contiguous() if b_mn else b
    out = gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out_dtype=torch.float32)
    assert _rel_err(out, ref) < 2e-3
    out16 = gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn)
    assert _rel_err(out16, ref) < 1e-2
    acc = torch.ones(m, n, device="cuda", dtype=torch.float32)
    gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out=acc, accumulate=True)
    assert _rel_err(acc, ref + 1) < 2e-3
    torch.cuda.synchronize()
    assert _native().read_status(True) == 0


def test_gemm_strided_views() -> None:
    from priml_b200.ops.functional import gemm

    big = torch.randn(512, 3 * 256, device="cuda", dtype=torch.bfloat16)
    a = big[:, 256:512]  # row stride 768
    b = torch.randn(384, 256, device="cuda", dtype=torch.bfloat16)
    out = gemm(a, b, out_dtype=torch.float32)
    assert _rel_err(out, a.float() @ b.float().T) < 2e-3


@pytest.mark.parametrize("m,h,k", [(256, 256, 128), (333, 384, 256), (1024, 1024, 512)])
def test_gemm_swiglu(m: int, h: int, k: int) -> None:
    torch.manual_seed(1)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2 * h, k, device="cuda", dtype=torch.bfloat16) / math.sqrt(k)
    hh = torch.empty(m, h, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(m, 2 * h, device="cuda", dtype=torch.bfloat16)
    _native().gemm_swiglu(x, w, hh, gu)
    ref_gu = x.float() @ w.float().T
    g, u = ref_gu.chunk(2, dim=-1)
    assert _rel_err(gu, ref_gu) < 1e-2
    assert _rel_err(hh, F.silu(g) * u) < 2e-2


def test_linear_autograd_matches_fp32() -> None:
    from priml_b200.ops import functional as fn

    torch.manual_seed(2)
    x = torch.randn(4, 96, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(768, 512, device="cuda", dtype=torch.float32, requires_grad=True)
    y = fn.linear(x, w)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().to(torch.bfloat16).float().requires_grad_()
    yr = xr @ wr.T
    yr.backward(gy.float())
    assert _rel_err(y, yr) < 1e-2
    assert _rel_err(x.grad, xr.grad) < 1e-2
    assert _rel_err(w.grad, wr.grad) < 2e-3


def test_rmsnorm_fwd_bwd() -> None:
    from priml_b200.ops import functional as fn

    torch.manual_seed(3)
    for dtype in (torch.bfloat16, torch.float32):
        x = torch.randn(37, 2048, device="cuda", dtype=dtype, requires_grad=True)
        w = torch.randn(2048, device="cuda", dtype=torch.float32, requires_grad=True)
        y = fn.rms_norm(x, w, 1e-5)
        gy = torch.randn_like(y)
        y.backward(gy)
        xr = x.detach().float().requires_grad_()
        wr = w.detach().requires_grad_()
        yr = F.rms_norm(xr, (2048,), wr, 1e-5)
        yr.backward(gy.float())
        tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
        assert _rel_err(y, yr) < tol
        assert _rel_err(x.grad, xr.grad) < tol * 2
        assert _rel_err(w.grad, wr.grad) < 1e-3


@pytest.mark.parametrize("x_dtype,d_dtype", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                             (torch.float32, torch.float32), (torch.float32, None)])
@pytest.mark.parametrize("affine", [False, True])
def test_add_rmsnorm_matches_fp32(x_dtype, d_dtype, affine) -> None:  # noqa: ANN001
    """h = x + d and rmsnorm(h) in one kernel; the backward merges the residual gradient dh with
    the norm's and writes d's gradient in d's dtype."""
    from priml_b200.ops import functional as fn

    torch.manual_seed(5)
    x = torch.randn(300, 2048, device="cuda", dtype=x_dtype, requires_grad=True)
    d = None if d_dtype is None else torch.randn(300, 2048, device="cuda", dtype=d_dtype, requires_grad=True)
    w = torch.randn(2048, device="cuda", requires_grad=True) if affine else None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        h, y = fn.add_rms_norm(x, d, w, 1e-5)
    gh, gy = torch.randn_like(h), torch.randn_like(y)
    torch.autograd.backward([h, y], [gh, gy])

    xr = x.detach().float().requires_grad_()
    dr = None if d is None else d.detach().float().requires_grad_()
    wr = None if w is None else w.detach().requires_grad_()
    hr = xr if dr is None else xr + dr
    if h.dtype == torch.bfloat16:
        hr = hr.bfloat16().float()  # the kernel normalizes the stored (rounded) sum
    yr = F.rms_norm(hr, (2048,), wr, 1e-5)
    torch.autograd.backward([hr, yr], [gh.float(), gy.float()])
    assert h.dtype == (torch.float32 if torch.float32 in (x_dtype, d_dtype) else torch.bfloat16)
    assert _rel_err(h, hr) < 1e-2
    assert _rel_err(y, yr) < 1e-2
    assert x.grad.dtype == x_dtype and _rel_err(x.grad, xr.grad) < 2e-2
    if d is not None:
        assert d.grad.dtype == d_dtype and _rel_err(d.grad, dr.grad) < 2e-2
    if w is not None:
        assert _rel_err(w.grad, wr.grad) < 1e-2


def test_deferred_residual_blocks_match_plain_blocks() -> None:
    """A CausalLM whose blocks pass (stream, delta) pairs equals one that adds after every block."""
    from priml_b200.models.presets import dense_lm

    torch.manual_seed(0)
    model = dense_lm(vocab=512, d_model=256, n_layers=3, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
                     rope_theta=1e4).make().cuda()  # fmt: skip
    tokens = torch.randint(0, 512, (2, 128), device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        fused = model.hidden_states(tokens)
        x = model.embed(tokens)
        for block in model.blocks:
            x = block(x)
        plain = model.final_norm(x)
    assert _rel_err(fused, plain) < 1e-2


def test_rope_matches_reference() -> None:
    from priml_b200.ops import functional as fn
    from priml_b200.ops import reference

    torch.manual_seed(4)
    qkv = torch.randn(2, 64, 12, 64, device="cuda", dtype=torch.bfloat16)
    q, k = qkv[:, :, :8], qkv[:, :, 8:10]
    pos = torch.arange(64, device="cuda", dtype=torch.float32)
    inv = 1.0 / (5e5 ** (torch.arange(0, 64, 2, device="cuda").float() / 64))
    ang = pos[:, None] * inv[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    qo, ko = fn.rotary(q, k, cos, sin)
    assert torch.equal(qo, reference.rotate_half(q, cos, sin))
    assert torch.equal(ko, reference.rotate_half(k, cos, sin))


def test_swiglu_and_ce() -> None:
    from priml_b200.ops import functional as fn

    torch.manual_seed(5)
    gu = torch.randn(100, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    h = fn.swiglu(gu)
    g, u = gu.detach().float().chunk(2, -1)
    assert _rel_err(h, F.silu(g) * u) < 1e-2
    h.sum().backward()
    gr = gu.detach().float().requires_grad_()
    a, b = gr.chunk(2, -1)
    (F.silu(a) * b).sum().backward()
    assert _rel_err(gu.grad, gr.grad) < 2e-2

    hid = torch.randn(300, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(1000, 256, device="cuda") / 16).requires_grad_()
    t = torch.randint(0, 1000, (300,), device="cuda")
    t[5] = -100
    loss = fn.linear_cross_entropy(hid, w, t)
    loss.mean().backward()
    hr = hid.detach().float().requires_grad_()
    wr = w.detach().to(torch.bfloat16).float().requires_grad_()
    logits = (hr @ wr.T).to(torch.bfloat16).float()
    lr = F.cross_entropy(logits, t, reduction="none")
    lr.mean().backward()
    assert _rel_err(loss, lr) < 1e-2
    assert _rel_err(hid.grad, hr.grad) < 3e-2
    assert _rel_err(w.grad, wr.grad) < 3e-2


@pytest.mark.parametrize("cap", [None, 15.0, 4.0])
@pytest.mark.parametrize("v", [1000, 8200])
def test_softcapped_cross_entropy_matches_fp32(cap, v: int) -> None:  # noqa: ANN001
    """Logit-level and fused-linear CE, capped and uncapped, against fp32 torch on the same bf16 logits."""
    from priml_b200 import ops

    torch.manual_seed(11)
    logits = (torch.randn(257, v, device="cuda") * 6).to(torch.bfloat16).requires_grad_()
    t = torch.randint(0, v, (257,), device="cuda")
    t[3] = -100
    loss = ops.cross_entropy(logits, t, softcap=cap)
    (loss * torch.linspace(0.5, 1.5, 257, device="cuda")).sum().backward()
    lf = logits.detach().float().requires_grad_()
    z = cap * torch.tanh(lf / cap) if cap is not None else lf
    lr = F.cross_entropy(z, t, reduction="none")
    (lr * torch.linspace(0.5, 1.5, 257, device="cuda")).sum().backward()
    assert float((loss - lr).abs().max()) < 2e-3 * (1 + float(lr.abs().max()))
    assert loss[3] == 0 and logits.grad[3].abs().max() == 0
    assert _rel_err(logits.grad, lf.grad) < 1e-2

    hid = torch.randn(300, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(v, 256, device="cuda") / 4).requires_grad_()
    tt = torch.randint(0, v, (300,), device="cuda")
    loss = ops.linear_cross_entropy(hid, w, tt, softcap=cap)
    loss.mean().backward()
    hr = hid.detach().float().requires_grad_()
    wr = w.detach().to(torch.bfloat16).float().requires_grad_()
    zl = (hr @ wr.T).to(torch.bfloat16).float()
    zl = cap * torch.tanh(zl / cap) if cap is not None else zl
    lr = F.cross_entropy(zl, tt, reduction="none")
    lr.mean().backward()
    assert _rel_err(loss, lr) < 1e-2
    assert _rel_err(hid.grad, hr.grad) < 3e-2
    assert _rel_err(w.grad, wr.grad) < 3e-2


def test_adamw_plan_matches_reference() -> None:
    from priml_b200.ops import reference

    torch.manual_seed(6)
    shapes = [(1000,), (64, 300), (3,)]
    ps = [torch.randn(s, device="cuda") for s in shapes]
    gs = [torch.randn(s, device="cuda") for s in shapes]
    ms = [torch.zeros(s, device="cuda") for s in shapes]
    vs = [torch.zeros(s, device="cuda") for s in shapes]
    shadows = [torch.empty(s, device="cuda", dtype=torch.bfloat16) for s in shapes]
    rp = [p.clone() for p in ps]
    rm = [m.clone() for m in ms]
    rv = [v.clone() for v in vs]
    plan = _native().MultiTensorPlan(ps, gs, ms, vs, shadows, 4096)
    for step in (1, 2, 3):
        b1 = 1 - 0.9**step
        b2 = 1 - 0.95**step
        plan.adamw(3e-4, 0.9, 0.95, 1e-8, 0.1, b1, b2, None)
        reference.adamw_(rp, gs, rm, rv, step=step, lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
    for p, r, s in zip(ps, rp, shadows, strict=True):
        assert _rel_err(p, r) < 1e-5
        assert torch.equal(s, p.to(torch.bfloat16))
    norm, clip = plan.grad_norm_clip(1.0)
    ref = torch.sqrt(sum((g.float() ** 2).sum() for g in gs))
    assert abs(float(norm) - float(ref)) / float(ref) < 1e-4
    assert abs(float(clip) - min(1.0, 1.0 / (float(ref) + 1e-6))) < 1e-6


@pytest.mark.parametrize("m,c,h", [(256, 256, 512), (300, 384, 264), (1024, 512, 1024)])
def test_swiglu_mlp_fused_fwd_bwd(m: int, c: int, h: int) -> None:
    """Up-projection + SwiGLU + down-projection with both epilogue fusions vs fp32 autograd."""
    from priml_b200.ops import functional as fn

    torch.manual_seed(0)
    x = torch.randn(m, c, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    wu = (torch.randn(2 * h, c, device="cuda") / math.sqrt(c)).requires_grad_()
    wd = (torch.randn(c, h, device="cuda") / math.sqrt(h)).requires_grad_()
    y = fn.swiglu_mlp(x, wu, wd)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr = x.detach().float().requires_grad_()
    wur = wu.detach().clone().requires_grad_()
    wdr = wd.detach().clone().requires_grad_()
    g, u = (xr @ wur.t()).chunk(2, dim=-1)
    yr = (F.silu(g) * u) @ wdr.t()
    yr.backward(dy.float())
    assert _rel_err(y, yr) < 2e-2
    assert _rel_err(x.grad, xr.grad) < 3e-2
    assert _rel_err(wu.grad, wur.grad) < 3e-2
    assert _rel_err(wd.grad, wdr.grad) < 3e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("mode", ["reflect", "replicate", "constant"])
def test_fused_augmentation_matches_torch_path(dtype: torch.dtype, mode: str) -> None:
    from priml_b200.data.augmentation_gpu import draw, pad_crop_flip

    torch.manual_seed(0)
    img = torch.randn(16, 3, 32, 32, device="cuda").to(dtype)
    d = draw(16, 32, 32, 4, None, img.device)
    fused = pad_crop_flip(img, 32, pad=4, pad_mode=mode, cutout_size=8, draws=d)
    ref = pad_crop_flip(img.cpu().float(), 32, pad=4, pad_mode=mode, cutout_size=8,
                        draws=type(d)(*(t.cpu() if t is not None else None for t in d)))  # fmt: skip
    assert torch.equal(fused.float().cpu(), ref.to(dtype).float())


@pytest.mark.parametrize("t,k,e,c,h", [(300, 2, 6, 256, 256), (1000, 6, 16, 512, 384)])
def test_grouped_swiglu_experts_fwd_bwd(t: int, k: int, e: int, c: int, h: int) -> None:
    import torch.nn.functional as F

    from priml_b200.ops import native
    from priml_b200.ops.grouped import grouped_swiglu_experts

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(t, c, device="cuda", generator=g).to(torch.bfloat16).requires_grad_()
    up = (torch.randn(e, 2 * h, c, device="cuda", generator=g) / c**0.5).requires_grad_()
    down = (torch.randn(e, c, h, device="cuda", generator=g) / h**0.5).requires_grad_()
    idx = torch.randint(0, e - 1, (t, k), device="cuda", generator=g)  # the last expert gets no rows
    w = torch.rand(t, k, device="cuda", generator=g)
    y = grouped_swiglu_experts(x, w, idx, up, down)
    gy = torch.randn(t, c, device="cuda", generator=g).to(torch.bfloat16)
    dx, dup, ddown = torch.autograd.grad(y, (x, up, down), gy)
    # fp32 oracle over the same bf16-rounded operands
    xf, upf, downf = x.detach().float(), up.detach().to(torch.bfloat16).float(), down.detach().to(torch.bfloat16).float()
    xf.requires_grad_()
    upf.requires_grad_()
    downf.requires_grad_()
    ref = torch.zeros(t, c, device="cuda")
    for ei in range(e):
        sel = (idx == ei).nonzero()
        if sel.numel() == 0:
            continue
        ti, j = sel[:, 0], sel[:, 1]
        gate, u = F.linear(xf[ti], upf[ei]).chunk(2, dim=-1)
        out = F.linear(F.silu(gate) * u, downf[ei]) * w[ti, j].unsqueeze(-1)
        ref = ref.index_add(0, ti, out)
    rx, rup, rdown = torch.autograd.grad(ref, (xf, upf, downf), gy.float())
    assert _rel_err(y, ref) < 2e-2
    assert _rel_err(dx, rx) < 3e-2
    assert _rel_err(dup, rup) < 3e-2
    assert _rel_err(ddown, rdown) < 3e-2
    assert float(dup[e - 1].abs().max()) == 0.0 and float(ddown[e - 1].abs().max()) == 0.0
    assert int(native().read_status(True)) == 0


@pytest.mark.parametrize("a_mn,b_mn", LAYOUTS)
@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (304, 520, 200), (1024, 2048, 512), (768, 3072, 768)])
def test_gemm_scaled_add_epilogue(a_mn: bool, b_mn: bool, m: int, n: int, k: int) -> None:
    """C = alpha * A @ B^T + beta * X against fp32 torch on the same bf16 operands."""
    torch.manual_seed(m + n + k)
    a = torch.randn(k, m, device="cuda").to(torch.bfloat16) if a_mn else torch.randn(m, k, device="cuda").to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda").to(torch.bfloat16) if b_mn else torch.randn(n, k, device="cuda").to(torch.bfloat16)
    x = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _native().gemm_axpby(a, b, x, c, a_mn, b_mn, -0.75, 1.5)
    af = a.float().T if a_mn else a.float()
    bf = b.float() if b_mn else b.float().T
    ref = -0.75 * (af @ bf) + 1.5 * x.float()
    assert _rel_err(c, ref) < 1e-2


@pytest.mark.parametrize("a_mn,b_mn", LAYOUTS)
@pytest.mark.parametrize("scaled", [False, True])
def test_gemm_batched_matches_fp32(a_mn: bool, b_mn: bool, scaled: bool) -> None:
    """One launch over a stack of products, plain and scaled-add epilogues."""
    torch.manual_seed(int(a_mn) + 2 * int(b_mn) + 4 * int(scaled))
    bsz, m, n, k = 3, 512, 256, 192
    a = torch.randn(bsz, k, m, device="cuda").to(torch.bfloat16) if a_mn else torch.randn(bsz, m, k, device="cuda").to(torch.bfloat16)
    b = torch.randn(bsz, k, n, device="cuda").to(torch.bfloat16) if b_mn else torch.randn(bsz, n, k, device="cuda").to(torch.bfloat16)
    x = torch.randn(bsz, m, n, device="cuda").to(torch.bfloat16)
    c = torch.empty(bsz, m, n, device="cuda", dtype=torch.bfloat16)
    if scaled:
        _native().gemm_batched(a, b, c, a_mn, b_mn, x, 0.5, -2.0)
    else:
        _native().gemm_batched(a, b, c, a_mn, b_mn)
    af = a.float().transpose(1, 2) if a_mn else a.float()
    bf = b.float() if b_mn else b.float().transpose(1, 2)
    ref = af @ bf
    if scaled:
        ref = 0.5 * ref - 2.0 * x.float()
    for i in range(bsz):
        assert _rel_err(c[i], ref[i]) < 1e-2, i


@pytest.mark.parametrize("shape", [(4, 768, 3072), (2, 2048, 512), (1, 1024, 1024), (3, 392, 520), (3, 300, 200)])
def test_newton_schulz_chain_matches_fp32(shape: tuple[int, ...]) -> None:
    """The tcgen05 Polar-Express chain (wide, tall, square, and a shape the torch path takes)
    against the same polynomial in fp32; its output is near-orthogonal."""
    from priml_b200.math.numeric import POLAR_EXPRESS_COEFFICIENTS
    from priml_b200.ops.orthogonalize import newton_schulz_reference, newton_schulz_steps

    torch.manual_seed(sum(shape))
    x = torch.randn(*shape, device="cuda")
    y = (x / (x.norm(dim=(-2, -1), keepdim=True) * 1.02 + 1e-6)).to(torch.bfloat16)
    out = newton_schulz_steps(y, POLAR_EXPRESS_COEFFICIENTS)
    ref = newton_schulz_reference(y.float(), POLAR_EXPRESS_COEFFICIENTS)
    assert out.shape == y.shape and out.dtype == torch.bfloat16
    assert _rel_err(out, ref) < 6e-2
    sv = torch.linalg.svdvals(out.float())
    assert float(sv.max()) < 1.3 and float(sv.median()) > 0.7
