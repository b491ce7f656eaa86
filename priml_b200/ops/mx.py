"""MXFP8 linear layers: E4M3 values with one E8M0 power-of-two scale per 32
elements along each GEMM's contraction dimension (OCP Microscaling v1.0).

Every GEMM of a linear layer's step runs in MXFP8 with blocks along its own
contraction dimension, so each operand is quantized for the GEMM that reads it:

* forward ``y = x W^T``: ``x`` and ``W`` in blocks along K;
* dgrad ``dx = dy W``: ``dy`` along N (its rows), ``W`` along N (stored
  transposed, ``[K, N]``);
* wgrad ``dW = dy^T x``: ``dy`` and ``x`` along the tokens (stored transposed),
  or in bf16 for the ``rowwise_gw_hp`` recipe.

On CUDA the quantizers and the block-scaled tcgen05 GEMM are ``mxfp8.cu``; the
fp32 accumulation and the scale application happen inside the tensor core.
Elsewhere (and as the test oracle) the same numbers come from
:func:`mx_quantize_ref` and a quantize-dequantize matmul.
"""

from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["mx_dequantize_ref", "mx_fake_quant", "mx_linear", "mx_quantize_ref", "mx_supported"]

_E4M3_MAX = 448.0


def mx_quantize_ref(x: Tensor) -> tuple[Tensor, Tensor]:
    """Reference MXFP8 quantization along the last dim (a multiple of 32).

    Returns ``(q, e)``: ``q`` float8_e4m3fn of ``x``'s shape and ``e`` the int32
    shared exponents ``[..., K / 32]`` (the E8M0 byte is ``e + 127``).
    """
    *lead, k = x.shape
    xb = x.float().reshape(*lead, k // 32, 32)
    amax = xb.abs().amax(-1)
    field = (amax.view(torch.int32) >> 23) & 0xFF
    e = torch.where(field == 0, torch.full_like(field, -127), field - 127) - 8
    e = e.clamp(-127, 127)
    scaled = xb * torch.ldexp(torch.ones_like(amax), -e).unsqueeze(-1)
    q = scaled.clamp(-_E4M3_MAX, _E4M3_MAX).to(torch.float8_e4m3fn)
    return q.reshape(*lead, k), e.to(torch.int32)


def mx_dequantize_ref(q: Tensor, e: Tensor) -> Tensor:
    *lead, k = q.shape
    v = q.float().reshape(*lead, k // 32, 32) * torch.ldexp(torch.ones_like(e, dtype=torch.float32), e).unsqueeze(-1)
    return v.reshape(*lead, k)


def mx_fake_quant(x: Tensor, dim: int = -1) -> Tensor:
    """``dequantize(quantize(x))`` with 32-element blocks along ``dim`` (fp32 result)."""
    xt = x.movedim(dim, -1)
    return mx_dequantize_ref(*mx_quantize_ref(xt)).movedim(-1, dim)


def mx_supported(m: int, n: int, k: int) -> bool:
    """Shapes the native path takes: every contraction dimension a multiple of 32."""
    return m % 32 == 0 and n % 32 == 0 and k % 32 == 0 and m > 0


class _WeightCache:
    """Quantized copies of a bf16 weight, reused while the weight is unchanged."""

    __slots__ = ("key", "rows", "cols")

    def __init__(self) -> None:
        self.key: tuple | None = None
        self.rows: tuple[Tensor, Tensor] | None = None
        self.cols: tuple[Tensor, Tensor] | None = None


def _weight_q(weight: Tensor, w16: Tensor, transpose: bool) -> tuple[Tensor, Tensor]:
    from priml_b200.ops import native

    root = weight._base if weight._base is not None else weight  # noqa: SLF001
    cache = getattr(root, "_pb_mx", None)
    key = (root._version, w16.data_ptr(), tuple(w16.shape))  # noqa: SLF001
    if cache is None:
        cache = _WeightCache()
        try:
            root._pb_mx = cache  # noqa: SLF001
        except (AttributeError, RuntimeError):
            return tuple(native().mx_quantize(w16, transpose))  # type: ignore[return-value]
    if cache.key != key:
        cache.key, cache.rows, cache.cols = key, None, None
    if transpose:
        if cache.cols is None:
            cache.cols = tuple(native().mx_quantize(w16, True))  # type: ignore[assignment]
        return cache.cols  # type: ignore[return-value]
    if cache.rows is None:
        cache.rows = tuple(native().mx_quantize(w16, False))  # type: ignore[assignment]
    return cache.rows  # type: ignore[return-value]


class _MXLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, wgrad_hp: bool) -> Tensor:  # type: ignore[override]
        from priml_b200.ops import native
        from priml_b200.ops.functional import _as_bf16_2d, bf16_shadow

        n = native()
        x2 = _as_bf16_2d(x).contiguous()
        w16 = bf16_shadow(weight).contiguous()
        qx, sx = n.mx_quantize(x2, False)
        qw, sw = _weight_q(weight, w16, False)
        y = torch.empty(x2.shape[0], w16.shape[0], device=x.device, dtype=torch.bfloat16)
        n.mx_gemm(qx, sx, qw, sw, y, 0)
        ctx.save_for_backward(x2, w16)
        ctx.weight, ctx.wgrad_hp, ctx.x_shape, ctx.x_dtype = weight, wgrad_hp, x.shape, x.dtype
        return y.view(*x.shape[:-1], w16.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        from priml_b200.ops import native
        from priml_b200.ops.functional import _as_bf16_2d, grad_sink, wgrad

        n = native()
        x2, w16 = ctx.saved_tensors
        dy2 = _as_bf16_2d(dy).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            qdy, sdy = n.mx_quantize(dy2, False)  # blocks along N
            qwt, swt = _weight_q(ctx.weight, w16, True)  # W^T [K, N], blocks along N
            dx = torch.empty(x2.shape[0], w16.shape[1], device=dy.device, dtype=torch.bfloat16)
            n.mx_gemm(qdy, sdy, qwt, swt, dx, 0)
            dx = dx.view(ctx.x_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            weight = ctx.weight
            if ctx.wgrad_hp:
                dw = wgrad(weight, dy2, x2, weight.dtype)
            else:
                qdyt, sdyt = n.mx_quantize(dy2, True)  # dy^T [N, M], blocks along tokens
                qxt, sxt = n.mx_quantize(x2, True)  # x^T [K, M]
                sink = grad_sink(weight)
                if sink is not None and weight.is_contiguous():
                    acc = sink.begin(weight)
                    out = sink.region(weight).view(w16.shape[0], w16.shape[1])
                    n.mx_gemm(qdyt, sdyt, qxt, sxt, out, 2 if acc else 1)
                else:
                    out = torch.empty(w16.shape[0], w16.shape[1], device=dy.device, dtype=torch.float32)
                    n.mx_gemm(qdyt, sdyt, qxt, sxt, out, 1)
                    dw = out if weight.dtype == torch.float32 else out.to(weight.dtype)
        return dx, dw, None


class _MXLinearRef(torch.autograd.Function):
    """Quantize-dequantize path with the native path's numerics (any device)."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, wgrad_hp: bool) -> Tensor:  # type: ignore[override]
        x2 = x.reshape(-1, x.shape[-1])
        y = mx_fake_quant(x2, -1) @ mx_fake_quant(weight.float(), -1).t()
        ctx.save_for_backward(x2, weight)
        ctx.wgrad_hp, ctx.x_shape = wgrad_hp, x.shape
        return y.to(x.dtype).view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, weight = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).float()
        dx = (mx_fake_quant(dy2, -1) @ mx_fake_quant(weight.float(), 0)).to(x2.dtype).view(ctx.x_shape)
        if ctx.wgrad_hp:
            dw = dy2.t() @ x2.float()
        else:
            dw = mx_fake_quant(dy2, 0).t() @ mx_fake_quant(x2.float(), 0)
        return dx, dw.to(weight.dtype), None


def mx_linear(x: Tensor, weight: Tensor, *, wgrad_high_precision: bool = False) -> Tensor:
    """``x @ weight^T`` with every GEMM of its step in MXFP8 (bias-free)."""
    from priml_b200 import ops

    m = x.numel() // x.shape[-1] if x.shape[-1] else 0
    n, k = weight.shape
    if ops.use_native(x, weight):
        if mx_supported(m, n, k):
            return _MXLinear.apply(x, weight, wgrad_high_precision)
        return ops.linear(x, weight)  # shapes outside MX blocks stay bf16
    if mx_supported(m, n, k):
        return _MXLinearRef.apply(x, weight, wgrad_high_precision)
    return torch.nn.functional.linear(x, weight.to(x.dtype))
