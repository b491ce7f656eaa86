"""Hot ops: hand-written sm_100a kernels on CUDA, pure-torch oracles elsewhere.

Every public op here dispatches on the device of its inputs:

* CUDA tensors run the in-tree extension ``priml_b200.ops._C`` (tcgen05/TMA
  GEMMs, attention, fused norm/rope/CE/optimizer kernels). When the extension
  is missing on a CUDA device the op raises -- there is no silent fallback.
* CPU tensors (and ``PRIML_B200_REFERENCE=1``) run :mod:`priml_b200.ops.reference`.
"""

from __future__ import annotations

import os

import torch
from torch import Tensor

from priml_b200.ops import reference
from priml_b200.ops._loader import native, native_available

__all__ = [
    "adamw_",
    "add_rms_norm",
    "attention",
    "cross_entropy",
    "decode_attention",
    "grouped_swiglu_experts",
    "grouped_swiglu_mlp",
    "mla_decode",
    "linear",
    "linear_cross_entropy",
    "linear_swiglu",
    "native",
    "native_available",
    "reference",
    "reference_forced",
    "rms_norm",
    "rotary",
    "swiglu",
    "swiglu_mlp",
    "use_native",
]


def use_native(*tensors: Tensor | None) -> bool:
    """True when these tensors should take the CUDA kernel path."""
    if os.environ.get("PRIML_B200_REFERENCE", "0") == "1":
        return False
    if any(t is not None and type(t).__name__ == "DTensor" for t in tensors):
        return False  # DTensor dispatch (tensor parallel on the decomposed path)
    return any(t is not None and t.is_cuda for t in tensors)


def reference_forced() -> bool:
    """True when ``PRIML_B200_REFERENCE=1`` pins every op to the torch oracle."""
    return os.environ.get("PRIML_B200_REFERENCE", "0") == "1"


def _compute_dtype(x: Tensor) -> torch.dtype:
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype


def linear(x: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    """``x @ weight.T (+ bias)``; weight ``[N, K]`` in its master dtype."""
    if use_native(x, weight) and _compute_dtype(x) == torch.bfloat16:
        from priml_b200.ops import functional

        return functional.linear(x, weight, bias)
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.nn.functional.linear(x, weight, bias)
    return reference.linear(x, weight, bias)


def rms_norm(x: Tensor, weight: Tensor | None, eps: float | None) -> Tensor:
    if use_native(x) and _compute_dtype(x) in (torch.bfloat16, torch.float32):
        from priml_b200.ops import functional

        return functional.rms_norm(x, weight, eps)
    return reference.rms_norm(x, weight, eps)


def add_rms_norm(x: Tensor, d: Tensor | None, weight: Tensor | None, eps: float | None) -> tuple[Tensor, Tensor]:
    """Residual add fused into RMSNorm: ``h = x + d`` (``x`` when ``d`` is None) and ``rmsnorm(h)``."""
    fusable = (
        x.shape[-1] % 8 == 0
        and x.dtype in (torch.bfloat16, torch.float32)
        and (d is None or (d.dtype in (torch.bfloat16, torch.float32) and d.shape == x.shape))
    )
    if fusable and use_native(x, d) and _compute_dtype(x) in (torch.bfloat16, torch.float32):
        from priml_b200.ops import functional

        return functional.add_rms_norm(x, d, weight, eps)
    h = x if d is None else x + d
    return h, reference.rms_norm(h, weight, eps)


def rotary(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor) -> tuple[Tensor, Tensor]:
    """Half-split RoPE of ``[B, S, H, D]`` q/k with ``[S, 1, D/2]`` fp32 factors."""
    if use_native(q) and q.dtype == torch.bfloat16 and cos.shape[-1] * 2 == q.shape[-1]:
        from priml_b200.ops import functional

        return functional.rotary(q, k, cos, sin)
    return reference.rotate_half(q, cos, sin), reference.rotate_half(k, cos, sin)


def attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    *,
    causal: bool = True,
    scale: float | None = None,
    window: int | None = None,
) -> Tensor:
    """Flash attention over ``[B, S, H, D]`` with native GQA (no K/V expansion)."""
    if use_native(q):
        from priml_b200.ops import functional

        if functional.attention_supported(q, k, v):
            return functional.attention(q, k, v, causal=causal, scale=scale, window=window)
    return reference.attention(q, k, v, causal=causal, scale=scale, window=window)


def linear_swiglu(x: Tensor, up_weight: Tensor) -> Tensor:
    """``silu(x @ Wg^T) * (x @ Wu^T)`` for ``up_weight = [Wg; Wu]`` (``[2H, C]``)."""
    if use_native(x) and _compute_dtype(x) == torch.bfloat16 and up_weight.shape[0] % 16 == 0 and x.shape[-1] % 8 == 0:
        from priml_b200.ops import functional

        return functional.linear_swiglu(x, up_weight)
    return swiglu(linear(x, up_weight))


def swiglu_mlp(x: Tensor, up_weight: Tensor, down_weight: Tensor) -> Tensor:
    """``down(silu(x Wg^T) * (x Wu^T))`` for ``up_weight = [Wg; Wu]`` ([2H, C]) and ``down_weight`` [C_out, H]."""
    if (
        use_native(x)
        and _compute_dtype(x) == torch.bfloat16
        and up_weight.shape[0] % 16 == 0
        and x.shape[-1] % 8 == 0
        and down_weight.shape[0] % 8 == 0
    ):
        from priml_b200.ops import functional

        return functional.swiglu_mlp(x, up_weight, down_weight)
    return linear(swiglu(linear(x, up_weight)), down_weight)


def swiglu(gate_up: Tensor) -> Tensor:
    if use_native(gate_up) and gate_up.dtype == torch.bfloat16:
        from priml_b200.ops import functional

        return functional.swiglu(gate_up)
    return reference.swiglu(gate_up)


def mla_decode(q: Tensor, c_kv: Tensor, k_pe: Tensor, *, scale: float, lengths: Tensor | None = None) -> Tensor:
    """Latent-space multi-head latent attention for one query token per sequence.

    ``q`` is ``[B, H, 576]``: the absorbed query ``q_nope @ W_UK`` (512) followed by the
    rotary query (64); ``c_kv [B, T, 512]`` and ``k_pe [B, T, 64]`` are the cached latent
    rows and shared rotary keys (any row / sequence strides with contiguous channels).
    Returns ``softmax(scale * q . [c_kv | k_pe]) @ c_kv`` per head, ``[B, H, 512]``; keys
    at or past ``lengths[b]`` are hidden. On CUDA (bf16) this is the tcgen05 kernel of
    ``ops/csrc/mla_decode.cu``.
    """
    if (
        use_native(q)
        and q.dtype == torch.bfloat16
        and c_kv.dtype == torch.bfloat16
        and k_pe.dtype == torch.bfloat16
        and q.shape[-1] == 576
        and c_kv.shape[-1] == 512
        and k_pe.shape[-1] == 64
        and c_kv.stride(-1) == 1
        and k_pe.stride(-1) == 1
        and all(st % 8 == 0 for st in (*c_kv.stride()[:-1], *k_pe.stride()[:-1]))
    ):
        return native().mla_decode(q.contiguous(), c_kv, k_pe, lengths, float(scale))
    return reference.mla_decode(q, c_kv, k_pe, scale=scale, lengths=lengths)


def decode_attention(
    q: Tensor,
    k_cache: Tensor,
    v_cache: Tensor,
    lengths: Tensor,
    *,
    scale: float | None = None,
    window: int | None = None,
) -> Tensor:
    """One query token per sequence against a KV cache with per-sequence lengths.

    ``q`` is ``[B, H, D]``; the caches are ``[B, Hkv, T, D]`` whose first
    ``lengths[b]`` rows are visible to sequence ``b`` (the query's own key
    included); query head ``h`` reads KV head ``h // (H / Hkv)``. ``window``
    hides keys more than ``window`` positions behind the query. The lengths stay
    on the device, so a decode step that calls this needs no host sync and can be
    captured in a CUDA graph. Returns ``[B, H, D]``.
    """
    if scale is None:
        scale = q.shape[-1] ** -0.5
    if (
        use_native(q)
        and q.dtype == torch.bfloat16
        and k_cache.dtype == torch.bfloat16
        and q.shape[-1] in (64, 128)
        and v_cache.shape[-1] == q.shape[-1]
    ):
        return native().decode_attn(
            q.contiguous(), k_cache, v_cache, lengths.to(torch.int32).contiguous(), float(scale),
            -1 if window is None else int(window),
        )  # fmt: skip
    return reference.decode_attention(q, k_cache, v_cache, lengths, scale=float(scale), window=window)


def cross_entropy(logits: Tensor, targets: Tensor, *, ignore_index: int = -100, softcap: float | None = None) -> Tensor:
    """Unreduced token CE in fp32 of ``[..., V]`` logits, optionally soft-capped by ``softcap * tanh(x / softcap)``.

    bf16 CUDA logits with ``V % 8 == 0`` run the CE kernels (one read of the row for the
    log-sum-exp, one read and one write for the gradient).
    """
    if (
        use_native(logits)
        and logits.dtype == torch.bfloat16
        and logits.shape[-1] % 8 == 0
        and (softcap is None or softcap > 0)
    ):
        from priml_b200.ops import functional

        return functional.cross_entropy(logits, targets, ignore_index=ignore_index, softcap=softcap)
    return reference.cross_entropy(logits, targets, ignore_index=ignore_index, softcap=softcap)


def linear_cross_entropy(
    hidden: Tensor,
    weight: Tensor,
    targets: Tensor,
    *,
    ignore_index: int = -100,
    softcap: float | None = None,
) -> Tensor:
    """Unreduced CE of ``hidden @ weight.T`` in fp32, optionally soft-capped.

    On CUDA the bf16 logits are written once by the GEMM; the CE kernels read them
    for the log-sum-exp (with the cap applied on the fly) and overwrite them with
    d(logits) in the backward, so no fp32 or capped copy of the logits exists.
    """
    if use_native(hidden) and _compute_dtype(hidden) == torch.bfloat16:
        from priml_b200.ops import functional

        return functional.linear_cross_entropy(hidden, weight, targets, ignore_index=ignore_index, softcap=softcap)
    return reference.linear_cross_entropy(hidden, weight, targets, ignore_index=ignore_index, softcap=softcap)


def grouped_swiglu_mlp(x_sorted: Tensor, up_w: Tensor, down_w: Tensor, offsets: Tensor) -> Tensor:
    """Grouped SwiGLU experts over expert segments ``offsets[e]:offsets[e+1]`` (device-side
    offsets; on CUDA the segments must start on multiples of 128, as the padded plan lays them out)."""
    if use_native(x_sorted):
        from priml_b200.ops import grouped

        return grouped.grouped_swiglu_mlp(x_sorted, up_w, down_w, offsets)
    return reference.grouped_swiglu_mlp(x_sorted, up_w, down_w, offsets)


def grouped_swiglu_experts(x: Tensor, weights: Tensor, indices: Tensor, up_w: Tensor, down_w: Tensor) -> Tensor:
    """Routed SwiGLU experts: padded device-side dispatch, grouped expert MLP, weighted combine."""
    from priml_b200.ops import grouped

    return grouped.grouped_swiglu_experts(x, weights, indices, up_w, down_w)


def adamw_(
    params: list[Tensor],
    grads: list[Tensor],
    exp_avgs: list[Tensor],
    exp_avg_sqs: list[Tensor],
    **hyper: float,
) -> None:
    if params and use_native(params[0]):
        from priml_b200.ops import functional

        functional.adamw_(params, grads, exp_avgs, exp_avg_sqs, **hyper)
        return
    reference.adamw_(params, grads, exp_avgs, exp_avg_sqs, **hyper)  # type: ignore[arg-type]
