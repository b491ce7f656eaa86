"""Grouped SwiGLU experts over 128-row-aligned expert segments.

Dispatch places the (token, choice) slots of expert ``e`` in rows
``offsets[e] : offsets[e] + count_e`` of a padded buffer whose segments start on
multiples of 128 (zero rows fill the gaps), so every 128-row GEMM tile belongs
to one expert. The buffer capacity ``ceil128(T * k) + 128 * E`` is a static
bound, and the plan is built with device ops only, so a whole MoE layer runs
without a host synchronization (the reference loops over experts after a
``.tolist()``, ``priml/model/moe.py:373-414``).

On CUDA the expert MLP is six grouped tcgen05 GEMM launches per step
(``grouped_gemm.cu``): up projection with the SwiGLU epilogue, down projection,
and in backward the down dgrad with the SwiGLU-backward epilogue, the up dgrad
and one grouped weight-gradient launch per weight (the K loop of each expert
runs over its own row segment).
"""

from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["grouped_swiglu_experts", "grouped_swiglu_mlp", "padded_dispatch_plan", "padded_capacity"]


def padded_capacity(slots: int, num_experts: int) -> int:
    """Static row bound of the padded expert buffer for ``slots`` (token, choice) pairs."""
    return (slots + 127) // 128 * 128 + 128 * num_experts


def padded_dispatch_plan(indices: Tensor, num_experts: int) -> tuple[Tensor, Tensor, int]:
    """``(pos, offsets, capacity)`` for ``[T, k]`` expert indices.

    ``pos[s]`` is the padded-buffer row of slot ``s = t * k + j`` (stable by
    slot within each expert); ``offsets`` (int32 ``[E + 1]``) delimits the
    128-aligned expert segments. Device ops only.
    """
    flat = indices.reshape(-1)
    n = flat.numel()
    counts = torch.bincount(flat, minlength=num_experts)
    padded = (counts + 127) // 128 * 128
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64, device=flat.device)
    offsets[1:] = torch.cumsum(padded, 0)
    order = torch.argsort(flat, stable=True)
    sorted_e = flat[order]
    starts = torch.cumsum(counts, 0) - counts
    rank = torch.arange(n, device=flat.device) - starts[sorted_e]
    pos = torch.empty_like(flat)
    pos[order] = offsets[sorted_e] + rank
    return pos, offsets.to(torch.int32), padded_capacity(n, num_experts)


def _grad_into(param: Tensor, e_rows: int) -> tuple[Tensor | None, bool, Tensor | None]:
    """(fp32 destination view, accumulate?, grad-sink) for a stacked expert weight."""
    from priml_b200.ops.functional import grad_sink

    sink = grad_sink(param)
    if sink is None or not param.is_contiguous():
        return None, False, None
    acc = sink.begin(param)
    return sink.region(param).view(e_rows, -1), acc, sink


class _GroupedSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_pad: Tensor, up_w: Tensor, down_w: Tensor, offsets: Tensor) -> Tensor:  # type: ignore[override]
        from priml_b200.ops import native
        from priml_b200.ops.functional import bf16_shadow

        n = native()
        e, two_h, c = up_w.shape
        h_dim = two_h // 2
        up16 = bf16_shadow(up_w).reshape(e * two_h, c)
        down16 = bf16_shadow(down_w).reshape(e * c, h_dim)
        rows = x_pad.shape[0]
        h = torch.empty(rows, h_dim, device=x_pad.device, dtype=torch.bfloat16)
        gu = torch.empty(rows, two_h, device=x_pad.device, dtype=torch.bfloat16)
        n.grouped_gemm(x_pad, up16, h, offsets, False, 3, 0, two_h, gu, h_dim)
        y = torch.empty(rows, c, device=x_pad.device, dtype=torch.bfloat16)
        n.grouped_gemm(h, down16, y, offsets, False, 0, 0, c)
        ctx.save_for_backward(x_pad, h, gu, up16, down16, offsets)
        ctx.params = (up_w, down_w)
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        from priml_b200.ops import native

        n = native()
        x_pad, h, gu, up16, down16, offsets = ctx.saved_tensors
        up_w, down_w = ctx.params
        e, two_h, c = up_w.shape
        h_dim = two_h // 2
        dy = dy.to(torch.bfloat16).contiguous()
        rows = dy.shape[0]
        dgu = torch.empty(rows, two_h, device=dy.device, dtype=torch.bfloat16)
        n.grouped_gemm(dy, down16, dgu, offsets, True, 4, 0, c, gu, h_dim)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(rows, c, device=dy.device, dtype=torch.bfloat16)
            n.grouped_gemm(dgu, up16, dx, offsets, True, 0, 0, two_h)
        grads = []
        for param, a, b in ((up_w, dgu, x_pad), (down_w, dy, h)):
            e_rows = param.shape[0] * param.shape[1]
            dst, acc, sink = _grad_into(param, e_rows)
            if dst is not None:
                n.grouped_gemm(a, b, dst, offsets, True, 2 if acc else 1, 1, 0)
                grads.append(None)
            else:
                out = torch.empty(e_rows, param.shape[2], device=dy.device, dtype=torch.float32)
                n.grouped_gemm(a, b, out, offsets, True, 1, 1, 0)
                grads.append(out.view_as(param).to(param.dtype))
        return dx, grads[0], grads[1], None


def grouped_swiglu_mlp(x_pad: Tensor, up_w: Tensor, down_w: Tensor, offsets: Tensor) -> Tensor:
    """Expert SwiGLU MLP over a padded buffer: rows of segment ``e`` use ``up_w[e]`` ``[2H, C]`` and ``down_w[e]`` ``[C, H]``."""
    from priml_b200 import ops

    e, two_h, c = up_w.shape
    native_ok = (
        ops.use_native(x_pad)
        and c % 128 == 0
        and two_h % 256 == 0
        and x_pad.shape[0] % 128 == 0
        and e <= 1024
    )
    if native_ok:
        return _GroupedSwiGLU.apply(x_pad.to(torch.bfloat16).contiguous(), up_w, down_w, offsets)
    return ops.reference.grouped_swiglu_mlp(x_pad, up_w, down_w, offsets)


def grouped_swiglu_experts(x: Tensor, weights: Tensor, indices: Tensor, up_w: Tensor, down_w: Tensor) -> Tensor:
    """Routed expert output ``sum_j weights[t, j] * expert_{indices[t, j]}(x[t])`` for ``x [T, C]``."""
    t, k = indices.shape
    e = up_w.shape[0]
    pos, offsets, cap = padded_dispatch_plan(indices, e)
    tok = torch.arange(t, device=x.device).repeat_interleave(k)
    dtype = torch.bfloat16 if x.is_cuda else x.dtype
    src = x.index_select(0, tok).to(dtype)
    x_pad = torch.zeros(cap, x.shape[1], device=x.device, dtype=dtype).index_copy(0, pos, src)
    y_pad = grouped_swiglu_mlp(x_pad, up_w, down_w, offsets)
    y = y_pad.index_select(0, pos).float() * weights.reshape(-1, 1).float()
    return y.view(t, k, -1).sum(1).to(x.dtype)
