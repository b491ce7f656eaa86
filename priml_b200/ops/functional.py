"""Autograd wrappers over the sm_100a kernels (CUDA path of :mod:`priml_b200.ops`).

Weights keep their master dtype (fp32). GEMMs read a bf16 **shadow** of each
weight, cached on the parameter and invalidated by the parameter's version
counter; :class:`priml_b200.optimizers.FusedAdamW` rewrites the shadow in the
same kernel that updates the master weight, so steady-state training does no
separate cast pass. Weight gradients are produced in fp32 directly by the
wgrad GEMM epilogue.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200.ops._loader import native

__all__ = [
    "GradSink",
    "add_rms_norm",
    "attention",
    "attention_supported",
    "bf16_shadow",
    "check_status",
    "gemm",
    "grad_sink",
    "grouped_swiglu_mlp",
    "linear",
    "linear_cross_entropy",
    "linear_swiglu",
    "rms_norm",
    "rotary",
    "swiglu",
    "swiglu_mlp",
    "wgrad",
]


# --------------------------------------------------------------------------- shadows
def _root(t: Tensor) -> Tensor:
    return t._base if t._base is not None else t  # noqa: SLF001


def bf16_shadow(weight: Tensor) -> Tensor:
    """bf16 view of ``weight`` (which may itself be a view of a parameter)."""
    if weight.dtype == torch.bfloat16:
        return weight
    root = _root(weight)
    cached = getattr(root, "_pb_shadow", None)
    version = root._version  # noqa: SLF001
    if cached is None or cached[0] != version or cached[1].shape != root.shape or cached[1].device != root.device:
        with torch.no_grad():
            sh = root.detach().to(torch.bfloat16).contiguous() if root.is_contiguous() else root.detach().to(torch.bfloat16)
        cached = (version, sh)
        try:
            root._pb_shadow = cached  # noqa: SLF001
        except (AttributeError, RuntimeError):
            return weight.detach().to(torch.bfloat16)
    sh = cached[1]
    if weight is root:
        return sh
    if not root.is_contiguous():
        return weight.detach().to(torch.bfloat16)
    return sh.as_strided(weight.shape, weight.stride(), weight.storage_offset() - root.storage_offset())


def attach_shadow(param: Tensor) -> Tensor:
    """Create (or refresh) and return the bf16 shadow of a contiguous fp32 parameter."""
    return bf16_shadow(param)


def mark_shadow_fresh(param: Tensor) -> None:
    """Declare the cached shadow current after a kernel rewrote it in place.

    Caches derived from the old values (quantized MXFP8 copies) are dropped: the
    kernel bypassed the version counter their keys check.
    """
    cached = getattr(param, "_pb_shadow", None)
    if cached is not None:
        param._pb_shadow = (param._version, cached[1])  # noqa: SLF001
    forget_quantized(param)


def forget_quantized(param: Tensor) -> None:
    """Drop the quantized copies cached on a weight whose values a kernel rewrote in place."""
    if "_pb_mx" in getattr(param, "__dict__", {}):
        del param.__dict__["_pb_mx"]


class GradSink:
    """fp32 destination of one parameter's gradient inside a flat buffer.

    Sharded data parallelism registers one on each parameter
    (``param._pb_grad_sink``); weight-gradient GEMMs then write their fp32
    output straight into it (overwriting on the first contribution of an
    accumulation window, accumulating afterwards) and hand autograd ``None``.
    """

    __slots__ = ("buf", "fresh")

    def __init__(self, buf: Tensor) -> None:
        self.buf = buf
        self.fresh = False

    def region(self, view: Tensor) -> Tensor:
        """The part of the buffer that corresponds to ``view`` of the parameter."""
        off = view.storage_offset() - _root(view).storage_offset()
        return self.buf.as_strided(view.shape, view.stride(), self.buf.storage_offset() + off)

    def begin(self, view: Tensor) -> bool:
        """Prepare a write of ``view``'s gradient; returns True to accumulate, False to overwrite."""
        if self.fresh:
            return True
        self.fresh = True
        if view.numel() == self.buf.numel():
            return False
        self.buf.zero_()
        return True

    def deliver(self, view: Tensor, grad: Tensor) -> None:
        region = self.region(view)
        if self.begin(view):
            region.add_(grad)
        else:
            region.copy_(grad)


def grad_sink(weight: Tensor) -> GradSink | None:
    return getattr(_root(weight), "_pb_grad_sink", None)


def wgrad(weight: Tensor, dy2: Tensor, x2: Tensor, w_dtype: torch.dtype) -> Tensor | None:
    """Weight gradient ``dy2^T x2`` (fp32 accumulate); written into the
    parameter's :class:`GradSink` when it has one (returns None), else returned
    in the weight's dtype."""
    sink = grad_sink(weight)
    if sink is not None and weight.is_contiguous():
        acc = sink.begin(weight)
        out = sink.region(weight).view(dy2.shape[1], x2.shape[1])
        gemm(dy2, x2, a_mn=True, b_mn=True, out=out, accumulate=acc)
        return None
    dw = gemm(dy2, x2, a_mn=True, b_mn=True, out_dtype=torch.float32)
    return dw if w_dtype == torch.float32 else dw.to(w_dtype)


def check_status(reset: bool = True) -> int:
    """Error code of the last kernel wait that timed out on this device (0 = none)."""
    return int(native().read_status(reset))


# --------------------------------------------------------------------------- GEMM
def gemm(a: Tensor, b: Tensor, *, a_mn: bool = False, b_mn: bool = False, out: Tensor | None = None,
         out_dtype: torch.dtype = torch.bfloat16, accumulate: bool = False) -> Tensor:  # fmt: skip
    """``C (+)= A @ B^T`` with A ``[M,K]`` (or ``[K,M]`` if ``a_mn``), B ``[N,K]`` (or ``[K,N]``)."""
    m = a.shape[1] if a_mn else a.shape[0]
    n = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty(m, n, device=a.device, dtype=torch.float32 if accumulate else out_dtype)
        if accumulate:
            out.zero_()
    epi = 2 if accumulate else (0 if out.dtype == torch.bfloat16 else 1)
    native().gemm(a, b, out, a_mn, b_mn, epi)
    return out


def _as_bf16_2d(x: Tensor) -> Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) % 8 != 0) or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    return x2


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, bias: Tensor | None) -> Tensor:  # type: ignore[override]
        x2 = _as_bf16_2d(x)
        w16 = bf16_shadow(weight)
        y = gemm(x2, w16)
        if bias is not None:
            y.add_(bias.to(y.dtype))
        ctx.save_for_backward(x2, w16)
        ctx.weight = weight if grad_sink(weight) is not None else None
        ctx.has_bias = bias is not None
        ctx.w_dtype = weight.dtype
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        return y.view(*x.shape[:-1], w16.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, w16 = ctx.saved_tensors
        dy2 = _as_bf16_2d(dy)
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dy2, w16, b_mn=True).view(ctx.x_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            dw = wgrad(ctx.weight if ctx.weight is not None else w16, dy2, x2, ctx.w_dtype)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = dy2.float().sum(0)
        return dx, dw, db


_GEMV_ROWS = 16
"""At most this many rows without autograd (decode steps) take a library GEMV: a 2-CTA tcgen05
tile is 256 rows tall, so a handful of rows leaves most of every tile idle and a layer's few
output tiles cover only a few SMs, while the product is a plain memory-bound matrix-vector read."""


def linear(x: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    if x.shape[-1] % 8 != 0 or weight.shape[0] % 8 != 0:
        w = weight.to(torch.bfloat16)
        return F.linear(x.to(torch.bfloat16), w, None if bias is None else bias.to(torch.bfloat16))
    if not torch.is_grad_enabled() and x.numel() // x.shape[-1] <= _GEMV_ROWS:
        w16 = bf16_shadow(weight)
        return F.linear(x.to(torch.bfloat16), w16, None if bias is None else bias.to(torch.bfloat16))
    return _Linear.apply(x, weight, bias)


class _LinearSwiGLU(torch.autograd.Function):
    """``silu(x Wg^T) * (x Wu^T)`` with the product fused into the GEMM epilogue."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor) -> Tensor:  # type: ignore[override]
        x2 = _as_bf16_2d(x)
        w16 = bf16_shadow(weight)
        two_h = w16.shape[0]
        h = torch.empty(x2.shape[0], two_h // 2, device=x.device, dtype=torch.bfloat16)
        gu = torch.empty(x2.shape[0], two_h, device=x.device, dtype=torch.bfloat16)
        native().gemm_swiglu(x2, w16, h, gu)
        ctx.save_for_backward(x2, w16, gu)
        ctx.weight = weight if grad_sink(weight) is not None else None
        ctx.w_dtype = weight.dtype
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        return h.view(*x.shape[:-1], two_h // 2)

    @staticmethod
    def backward(ctx, dh: Tensor):  # type: ignore[override]
        x2, w16, gu = ctx.saved_tensors
        dgu = native().swiglu_bwd(gu, _as_bf16_2d(dh))
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dgu, w16, b_mn=True).view(ctx.x_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            dw = wgrad(ctx.weight if ctx.weight is not None else w16, dgu, x2, ctx.w_dtype)
        return dx, dw


def linear_swiglu(x: Tensor, weight: Tensor) -> Tensor:
    if not torch.is_grad_enabled() and x.numel() // x.shape[-1] <= _GEMV_ROWS:
        return swiglu(linear(x, weight))
    return _LinearSwiGLU.apply(x, weight)


class _SwiGLUMLP(torch.autograd.Function):
    """``down(silu(x Wg^T) * (x Wu^T))`` as one autograd node: the forward fuses
    the activation into the up-projection epilogue, the backward fuses the
    SwiGLU derivative into the epilogue of ``dy @ W_down`` (dh never exists)."""

    @staticmethod
    def forward(ctx, x: Tensor, w_up: Tensor, w_down: Tensor) -> Tensor:  # type: ignore[override]
        x2 = _as_bf16_2d(x)
        wu = bf16_shadow(w_up)
        wd = bf16_shadow(w_down)
        two_h = wu.shape[0]
        h = torch.empty(x2.shape[0], two_h // 2, device=x.device, dtype=torch.bfloat16)
        gu = torch.empty(x2.shape[0], two_h, device=x.device, dtype=torch.bfloat16)
        native().gemm_swiglu(x2, wu, h, gu)
        y = gemm(h, wd)
        ctx.save_for_backward(x2, wu, wd, gu, h)
        ctx.w_up = w_up if grad_sink(w_up) is not None else None
        ctx.w_down = w_down if grad_sink(w_down) is not None else None
        ctx.dtypes = (w_up.dtype, w_down.dtype)
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        return y.view(*x.shape[:-1], wd.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, wu, wd, gu, h = ctx.saved_tensors
        dy2 = _as_bf16_2d(dy)
        dgu = torch.empty_like(gu)
        native().gemm_swiglu_bwd(dy2, wd, gu, dgu)
        dx = dwu = dwd = None
        if ctx.needs_input_grad[2]:
            dwd = wgrad(ctx.w_down if ctx.w_down is not None else wd, dy2, h, ctx.dtypes[1])
        if ctx.needs_input_grad[0]:
            dx = gemm(dgu, wu, b_mn=True).view(ctx.x_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            dwu = wgrad(ctx.w_up if ctx.w_up is not None else wu, dgu, x2, ctx.dtypes[0])
        return dx, dwu, dwd


def swiglu_mlp(x: Tensor, w_up: Tensor, w_down: Tensor) -> Tensor:
    if not torch.is_grad_enabled() and x.numel() // x.shape[-1] <= _GEMV_ROWS:
        return linear(swiglu(linear(x, w_up)), w_down)
    return _SwiGLUMLP.apply(x, w_up, w_down)


# --------------------------------------------------------------------------- elementwise
def _eps(eps: float | None, x: Tensor) -> float:
    if eps is not None:
        return float(eps)
    dtype = torch.float32 if torch.is_autocast_enabled("cuda") else x.dtype
    return float(torch.finfo(dtype).eps)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor | None, eps: float, out_f32: bool) -> Tensor:  # type: ignore[override]
        xc = x.contiguous()
        y, rstd = native().rmsnorm_fwd(xc, weight, eps, out_f32)
        ctx.save_for_backward(xc, weight, rstd)
        ctx.x_f32 = x.dtype == torch.float32
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x, weight, rstd = ctx.saved_tensors
        dx, dw = native().rmsnorm_bwd(dy, x, weight, rstd, ctx.x_f32)
        sink = grad_sink(weight) if weight is not None and dw is not None else None
        if sink is not None:
            sink.deliver(weight, dw)
            dw = None
        elif weight is not None and dw is not None and dw.dtype != weight.dtype:
            dw = dw.to(weight.dtype)
        return dx, (dw if weight is not None else None), None, None


def rms_norm(x: Tensor, weight: Tensor | None, eps: float | None) -> Tensor:
    if x.shape[-1] % 8 != 0 or x.dtype not in (torch.bfloat16, torch.float32):
        return F.rms_norm(x, (x.shape[-1],), weight, eps)
    out_f32 = x.dtype == torch.float32 and not torch.is_autocast_enabled("cuda")
    return _RMSNorm.apply(x, weight, _eps(eps, x), out_f32)


class _AddRMSNorm(torch.autograd.Function):
    """``(h, y) = (x + d, rmsnorm(x + d))`` in one kernel; ``d`` may be ``None`` (then ``h`` is ``x``).

    The backward merges the two gradients that reach ``h`` -- along the residual stream and
    through the norm -- in the norm's backward kernel, and writes ``d``'s copy of that gradient
    in ``d``'s dtype, so neither the add nor its gradient costs a separate elementwise pass.
    """

    @staticmethod
    def forward(ctx, x: Tensor, d: Tensor | None, weight: Tensor | None, eps: float, out_f32: bool):  # type: ignore[override]
        ctx.set_materialize_grads(False)
        if d is None:
            h = x.contiguous()
            y, rstd = native().rmsnorm_fwd(h, weight, eps, out_f32)
        else:
            h, y, rstd = native().add_rmsnorm_fwd(x, d, weight, eps, out_f32)
        ctx.save_for_backward(h, weight, rstd)
        ctx.x_dtype = x.dtype
        ctx.d_dtype = None if d is None else d.dtype
        return h, y

    @staticmethod
    def backward(ctx, dh: Tensor | None, dy: Tensor | None):  # type: ignore[override]
        h, weight, rstd = ctx.saved_tensors
        if dy is None:
            if dh is None:
                return None, None, None, None, None
            dd = None if ctx.d_dtype is None else dh.to(ctx.d_dtype)
            return dh.to(ctx.x_dtype), dd, None, None, None
        dd_code = -1 if ctx.d_dtype is None else (1 if ctx.d_dtype == torch.float32 else 0)
        dx, dd, dw = native().add_rmsnorm_bwd(dy, h, weight, rstd, dh, ctx.x_dtype == torch.float32, dd_code)
        sink = grad_sink(weight) if weight is not None and dw is not None else None
        if sink is not None:
            sink.deliver(weight, dw)
            dw = None
        elif weight is not None and dw is not None and dw.dtype != weight.dtype:
            dw = dw.to(weight.dtype)
        return dx, (dd if ctx.d_dtype is not None else None), (dw if weight is not None else None), None, None


def add_rms_norm(x: Tensor, d: Tensor | None, weight: Tensor | None, eps: float | None) -> tuple[Tensor, Tensor]:
    """Residual add fused into RMSNorm: returns ``(x + d, rmsnorm(x + d))`` (``d=None``: ``(x, rmsnorm(x))``)."""
    out_f32 = x.dtype == torch.float32 and not torch.is_autocast_enabled("cuda")
    return _AddRMSNorm.apply(x, d, weight, _eps(eps, x), out_f32)


class _Rotary(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q: Tensor, k: Tensor, cos: Tensor, sin: Tensor) -> tuple[Tensor, Tensor]:  # type: ignore[override]
        c = cos.reshape(cos.shape[0], -1)
        s = sin.reshape(sin.shape[0], -1)
        ctx.save_for_backward(c, s)
        n = native()
        return n.rope(q, c, s, 1.0), n.rope(k, c, s, 1.0)

    @staticmethod
    def backward(ctx, dq: Tensor, dk: Tensor):  # type: ignore[override]
        c, s = ctx.saved_tensors
        n = native()
        return n.rope(dq.contiguous(), c, s, -1.0), n.rope(dk.contiguous(), c, s, -1.0), None, None


def rotary(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor) -> tuple[Tensor, Tensor]:
    if q.shape[-1] % 4 != 0 or cos.requires_grad or sin.requires_grad:
        from priml_b200.ops import reference

        return reference.rotate_half(q, cos, sin), reference.rotate_half(k, cos, sin)
    return _Rotary.apply(q, k, cos.float(), sin.float())


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu: Tensor) -> Tensor:  # type: ignore[override]
        guc = gu.contiguous()
        ctx.save_for_backward(guc)
        return native().swiglu_fwd(guc)

    @staticmethod
    def backward(ctx, dh: Tensor):  # type: ignore[override]
        (gu,) = ctx.saved_tensors
        return native().swiglu_bwd(gu, dh)


def swiglu(gu: Tensor) -> Tensor:
    if gu.shape[-1] % 16 != 0:
        g, u = gu.chunk(2, dim=-1)
        return F.silu(g) * u
    return _SwiGLU.apply(gu)


# --------------------------------------------------------------------------- attention
def attention_supported(q: Tensor, k: Tensor, v: Tensor) -> bool:
    return q.dtype in (torch.bfloat16, torch.float16) or torch.is_autocast_enabled("cuda")


def attention(q: Tensor, k: Tensor, v: Tensor, *, causal: bool, scale: float | None, window: int | None) -> Tensor:
    """``[B,S,H,D]`` flash attention with grouped KV heads."""
    from priml_b200.ops import flash as attn_mod

    return attn_mod.flash_attention(q, k, v, causal=causal, scale=scale, window=window)


# --------------------------------------------------------------------------- loss
class _LinearCE(torch.autograd.Function):
    """CE of ``hidden @ weight.T``: one bf16 logits buffer, fp32 log-sum-exp, d(logits) written in place.

    ``softcap`` > 0 bounds each logit by ``softcap * tanh(x / softcap)`` inside the
    CE kernels (``priml/model/softcap.py:89-94`` followed by the loss of
    ``priml/baselines/nanochat/train_step.py:43-79``), so the capped logits are
    never stored.
    """

    @staticmethod
    def forward(ctx, h: Tensor, weight: Tensor, targets: Tensor, ignore_index: int, softcap: float) -> Tensor:  # type: ignore[override]
        h2 = _as_bf16_2d(h)
        w16 = bf16_shadow(weight)
        logits = gemm(h2, w16)
        t = targets.reshape(-1)
        loss, lse = native().ce_fwd(logits, t, ignore_index, softcap)
        ctx.save_for_backward(h2, w16, logits, t, lse)
        ctx.weight = weight if grad_sink(weight) is not None else None
        ctx.ignore_index = ignore_index
        ctx.softcap = softcap
        ctx.h_shape = h.shape
        ctx.h_dtype = h.dtype
        ctx.w_dtype = weight.dtype
        return loss.view(targets.shape)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        h2, w16, logits, t, lse = ctx.saved_tensors
        gf = g.reshape(-1).float()
        if gf.stride(0) == 0:
            gf = gf[:1]
        # in place: logits -> dlogits
        native().ce_bwd(logits, t, lse, gf.contiguous(), logits, ctx.ignore_index, ctx.softcap)
        dh = dw = None
        if ctx.needs_input_grad[0]:
            dh = gemm(logits, w16, b_mn=True).view(ctx.h_shape)
            if ctx.h_dtype != torch.bfloat16:
                dh = dh.to(ctx.h_dtype)
        if ctx.needs_input_grad[1]:
            dw = wgrad(ctx.weight if ctx.weight is not None else w16, logits, h2, ctx.w_dtype)
        return dh, dw, None, None, None


def linear_cross_entropy(
    hidden: Tensor, weight: Tensor, targets: Tensor, *, ignore_index: int = -100, softcap: float | None = None
) -> Tensor:
    if weight.shape[0] % 8 != 0 or hidden.shape[-1] % 8 != 0 or (softcap is not None and not softcap > 0):
        from priml_b200.ops import reference

        return reference.linear_cross_entropy(hidden, weight, targets, ignore_index=ignore_index, softcap=softcap)
    return _LinearCE.apply(hidden, weight, targets, ignore_index, float(softcap or 0.0))


class _CE(torch.autograd.Function):
    """Token CE over given bf16 logits (optionally soft-capped); d(logits) comes back in bf16."""

    @staticmethod
    def forward(ctx, logits: Tensor, targets: Tensor, ignore_index: int, softcap: float) -> Tensor:  # type: ignore[override]
        l2 = logits.reshape(-1, logits.shape[-1])
        if l2.stride(-1) != 1 or l2.stride(0) % 8 != 0:
            l2 = l2.contiguous()
        t = targets.reshape(-1)
        loss, lse = native().ce_fwd(l2, t, ignore_index, softcap)
        ctx.save_for_backward(l2, t, lse)
        ctx.ignore_index, ctx.softcap, ctx.shape = ignore_index, softcap, logits.shape
        return loss.view(targets.shape)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        l2, t, lse = ctx.saved_tensors
        gf = g.reshape(-1).float()
        if gf.stride(0) == 0:
            gf = gf[:1]
        d = torch.empty_like(l2)
        native().ce_bwd(l2, t, lse, gf.contiguous(), d, ctx.ignore_index, ctx.softcap)
        return d.view(ctx.shape), None, None, None


def cross_entropy(logits: Tensor, targets: Tensor, *, ignore_index: int = -100, softcap: float | None = None) -> Tensor:
    return _CE.apply(logits, targets, ignore_index, float(softcap or 0.0))


# --------------------------------------------------------------------------- MoE
def grouped_swiglu_mlp(x_sorted: Tensor, up_w: Tensor, down_w: Tensor, offsets: Tensor) -> Tensor:
    from priml_b200.ops import grouped

    return grouped.grouped_swiglu_mlp(x_sorted, up_w, down_w, offsets)


# --------------------------------------------------------------------------- optimizer
def adamw_(params, grads, exp_avgs, exp_avg_sqs, **hyper) -> None:  # noqa: ANN001
    from priml_b200.ops import reference

    reference.adamw_(params, grads, exp_avgs, exp_avg_sqs, **hyper)


_ = math
