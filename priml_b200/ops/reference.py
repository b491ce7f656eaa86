"""Pure-torch oracles for every hand-written kernel.

These are the semantics the CUDA kernels reproduce; tests compare the kernels
against them computed in fp32. They are also the CPU execution path (the
reference framework itself runs these ops through ATen:
``priml/model/norm.py:36-74``, ``priml/model/rope.py:348-387``,
``priml/model/attention.py:107-193``, ``priml/model/swiglu.py:190-213``,
``priml/baselines/nanochat/train_step.py:43-79``,
``priml/optimizers/fused_adamw.py:42-83``).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor


def linear(x: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    w = weight.to(x.dtype)
    return F.linear(x, w, None if bias is None else bias.to(x.dtype))


def rms_norm(x: Tensor, weight: Tensor | None, eps: float | None) -> Tensor:
    return F.rms_norm(x, (x.shape[-1],), weight, eps)


def rotate_half(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Half-split rotation in fp32, rounded once (HuggingFace convention)."""
    dtype = x.dtype
    x = x.float()
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half], x[..., half:]
    return torch.cat([x0 * cos - x1 * sin, x1 * cos + x0 * sin], dim=-1).to(dtype)


def attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    *,
    causal: bool = True,
    scale: float | None = None,
    window: int | None = None,
) -> Tensor:
    """``[B, S, H, D]`` x ``[B, T, Hkv, D]`` -> ``[B, S, H, Dv]``; grouped KV heads
    are shared by ``H // Hkv`` consecutive query heads. Causal masks are aligned
    bottom-right (query ``i`` sees keys ``<= T - S + i``); ``window`` limits the
    look-back to ``window`` keys (``key >= pos - window``)."""
    B, S, H, D = q.shape
    T, Hkv = k.shape[1], k.shape[2]
    g = H // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qf = q.float().transpose(1, 2)  # B H S D
    kf = k.float().transpose(1, 2).repeat_interleave(g, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(g, dim=1)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    if causal or window is not None:
        qi = torch.arange(S, device=q.device)[:, None] + (T - S)
        kj = torch.arange(T, device=q.device)[None, :]
        allowed = torch.ones(S, T, dtype=torch.bool, device=q.device)
        if causal:
            allowed &= kj <= qi
        if window is not None:
            allowed &= kj >= qi - window
        s = s.masked_fill(~allowed, float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    o = torch.matmul(p, vf)
    return o.transpose(1, 2).to(q.dtype)


def swiglu(gate_up: Tensor) -> Tensor:
    gate, up = gate_up.chunk(2, dim=-1)
    return F.silu(gate) * up


def decode_attention(
    q: Tensor, k_cache: Tensor, v_cache: Tensor, lengths: Tensor, *, scale: float, window: int | None = None
) -> Tensor:
    """fp32 oracle of the decode kernel: ``[B, H, D]`` queries over ``[B, Hkv, T, D]`` caches."""
    b, h, _ = q.shape
    hkv, t = k_cache.shape[1], k_cache.shape[2]
    kf = k_cache.float().repeat_interleave(h // hkv, dim=1)
    vf = v_cache.float().repeat_interleave(h // hkv, dim=1)
    s = torch.einsum("bhd,bhtd->bht", q.float(), kf) * scale
    pos = torch.arange(t, device=q.device)
    n = lengths.to(device=q.device, dtype=torch.long).clamp(0, t)[:, None]
    ok = pos[None, :] < n
    if window is not None:
        ok &= pos[None, :] >= n - 1 - window
    s = s.masked_fill(~ok[:, None, :], float("-inf"))
    p = torch.nan_to_num(s.softmax(dim=-1), nan=0.0)  # an empty row gives zeros
    return torch.einsum("bht,bhtd->bhd", p, vf).to(q.dtype)


def mla_decode(
    q: Tensor, c_kv: Tensor, k_pe: Tensor, *, scale: float, lengths: Tensor | None = None
) -> Tensor:
    """fp32 oracle of latent-space MLA decode: ``q [B, H, 576] = [q_abs | q_pe]`` over
    ``c_kv [B, T, 512]`` and ``k_pe [B, T, 64]``; returns the softmax-weighted latent rows ``[B, H, 512]``."""
    lat = c_kv.shape[-1]
    c = c_kv.float()
    s = (torch.einsum("bhl,btl->bht", q[..., :lat].float(), c)
         + torch.einsum("bhr,btr->bht", q[..., lat:].float(), k_pe.float())) * scale  # fmt: skip
    if lengths is not None:
        pos = torch.arange(c.shape[1], device=q.device)
        ok = pos[None, :] < lengths.to(device=q.device, dtype=torch.long)[:, None]
        s = s.masked_fill(~ok[:, None, :], float("-inf"))
    p = torch.nan_to_num(s.softmax(dim=-1), nan=0.0)
    return torch.einsum("bht,btl->bhl", p, c).to(q.dtype)


def cross_entropy(logits: Tensor, targets: Tensor, *, ignore_index: int = -100, softcap: float | None = None) -> Tensor:
    """Unreduced token cross-entropy computed in fp32."""
    lf = logits.float()
    if softcap is not None:
        lf = softcap * torch.tanh(lf / softcap)
    return F.cross_entropy(lf.reshape(-1, lf.shape[-1]), targets.reshape(-1), ignore_index=ignore_index, reduction="none").reshape(
        targets.shape
    )


def linear_cross_entropy(
    hidden: Tensor,
    weight: Tensor,
    targets: Tensor,
    *,
    ignore_index: int = -100,
    softcap: float | None = None,
) -> Tensor:
    logits = linear(hidden, weight)
    return cross_entropy(logits, targets, ignore_index=ignore_index, softcap=softcap)


def adamw_(
    params: list[Tensor],
    grads: list[Tensor],
    exp_avgs: list[Tensor],
    exp_avg_sqs: list[Tensor],
    *,
    step: int,
    lr: float,
    beta1: float,
    beta2: float,
    eps: float,
    weight_decay: float,
) -> None:
    """AdamW in the FusedAdamW operation order (``priml/optimizers/fused_adamw.py:42-83``):
    ``p *= 1 - lr*wd``; ``m = lerp(m, g, 1-b1)``; ``v = lerp(v, g*g, 1-b2)``;
    ``p -= m / (sqrt(v / bias2) + eps) * (lr / bias1)`` -- all in fp32."""
    bias1 = 1.0 - beta1**step
    bias2 = 1.0 - beta2**step
    with torch.no_grad():
        for p, g, m, v in zip(params, grads, exp_avgs, exp_avg_sqs, strict=True):
            g32 = g.float()
            p32 = p if p.dtype == torch.float32 else p.float()
            m32 = m if m.dtype == torch.float32 else m.float()  # moments of narrow parameters update in fp32
            v32 = v if v.dtype == torch.float32 else v.float()
            p32.mul_(1.0 - lr * weight_decay)
            m32.lerp_(g32, 1.0 - beta1)
            v32.lerp_(g32.square(), 1.0 - beta2)
            denom = (v32 / bias2).sqrt() + eps
            p32.sub_(m32 / denom * (lr / bias1))
            for lo, hi in ((p, p32), (m, m32), (v, v32)):
                if hi.data_ptr() != lo.data_ptr():
                    lo.copy_(hi)


def grouped_swiglu_mlp(x_sorted: Tensor, up_w: Tensor, down_w: Tensor, offsets: Tensor) -> Tensor:
    """Rows ``offsets[e]:offsets[e+1]`` through expert ``e``:
    ``down_w[e] @ swiglu(up_w[e] @ x)``; ``up_w [E, 2H, C]``, ``down_w [E, C, H]``.
    Rows past ``offsets[E]`` (padding of a padded buffer) come out zero."""
    bounds = offsets.tolist()
    pieces = []
    for e in range(up_w.shape[0]):
        lo, hi = bounds[e], bounds[e + 1]
        if hi > lo:
            pieces.append(linear(swiglu(linear(x_sorted[lo:hi], up_w[e])), down_w[e]))
    tail = x_sorted.shape[0] - bounds[-1]  # rows past the last segment (padded buffers)
    if tail > 0:
        pieces.append(x_sorted.new_zeros(tail, down_w.shape[1]))
    if not pieces:
        return x_sorted.new_zeros(0, down_w.shape[1])
    return torch.cat(pieces, dim=0)
