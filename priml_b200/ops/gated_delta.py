"""Chunked gated delta rule with the chunk scan on tcgen05 kernels (``csrc/gated_delta.cu``).

Counterpart of ``chunk_gated_delta_rule`` as ``priml/model/gated_delta_net.py:172-193``
calls it (``use_qk_l2norm_in_kernel=True``, no initial or final state).

Per value head the delta rule keeps a state ``H`` (``[dk, dv]``) and with
``alpha_t = exp(g_t)``:

    H_t = alpha_t (I - beta_t k_t k_t^T) H_{t-1} + beta_t k_t v_t^T,    o_t = H_t^T q_t

Chunks of C = 128 tokens split the work. With ``G`` the within-chunk cumulative sum of
``g`` (``gamma_t = exp(G_t)``) and ``A_ts = beta_t exp(G_t - G_s) k_s . k_t`` for s < t,
everything that does not depend on the running state is chunk-parallel:

    W  = (I + A)^-1 (beta gamma K)      Ut = (I + A)^-1 (beta V)
    Qg = gamma Q     Kr = exp(G_C - G) K     Mqk = tril(exp(G_t - G_s) Q K^T)     gC = gamma_C

(batched GEMMs and one batched triangular solve, differentiated by autograd). The rest is a
sequential scan over the chunks, ``U = Ut - W H``, ``O = Qg H + Mqk U``,
``H <- gC H + Kr^T U``, which runs in ``gdn_fwd`` / ``gdn_bwd`` (one CTA per batch-head,
state in TMEM). Its backward walks the chunks in reverse,
``dU = Mqk^T dO + Kr dH'``, ``dH = gC dH' + Qg^T dO - W^T dU``, and the gradients of the
chunk-parallel operands follow from the saved states as batched GEMMs (:class:`_Scan`).
:func:`scan_reference` / :func:`scan_reference_bwd` restate the two kernels in torch so the
algebra is checked on CPU against the token-by-token recurrence.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200.ops._loader import native

__all__ = ["CHUNK", "chunk_operands", "gated_delta_rule", "kernel_supported", "scan_reference", "scan_reference_bwd"]

CHUNK = 128


def kernel_supported(dk: int, dv: int) -> bool:
    """The scan kernels cover head widths dk = dv = 128."""
    return dk == CHUNK and dv == CHUNK


def _l2n(x: Tensor, eps: float = 1e-6) -> Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def scan_reference(w: Tensor, ut: Tensor, qg: Tensor, mqk: Tensor, kr: Tensor, gc: Tensor) -> tuple[Tensor, ...]:
    """The forward scan in torch (fp32): returns (O, entry states, U), like ``gdn_fwd``."""
    bh, n, C, dk = w.shape
    dv = ut.shape[-1]
    h = w.new_zeros(bh, dk, dv, dtype=torch.float32)
    outs, states, us = [], [], []
    for c in range(n):
        states.append(h)
        u = ut[:, c].float() - w[:, c].float() @ h
        outs.append(qg[:, c].float() @ h + mqk[:, c].float() @ u)
        us.append(u)
        h = gc[:, c, None, None] * h + kr[:, c].float().transpose(-1, -2) @ u
    return torch.stack(outs, 1), torch.stack(states, 1), torch.stack(us, 1)


def scan_reference_bwd(kr: Tensor, mqk: Tensor, do: Tensor, qg: Tensor, w: Tensor, gc: Tensor) -> tuple[Tensor, Tensor]:
    """The backward scan in torch (fp32): returns (dU, gradient of each chunk's exit state)."""
    bh, n, C, dk = kr.shape
    dv = do.shape[-1]
    dh = kr.new_zeros(bh, dk, dv, dtype=torch.float32)
    dus, dhs = [None] * n, [None] * n
    for c in reversed(range(n)):
        dhs[c] = dh
        du = mqk[:, c].float().transpose(-1, -2) @ do[:, c].float() + kr[:, c].float() @ dh
        dus[c] = du
        dh = gc[:, c, None, None] * dh + qg[:, c].float().transpose(-1, -2) @ do[:, c].float() - w[:, c].float().transpose(-1, -2) @ du
    return torch.stack(dus, 1), torch.stack(dhs, 1)


class _Scan(torch.autograd.Function):
    """The chunk scan: kernels on CUDA, :func:`scan_reference` elsewhere."""

    @staticmethod
    def forward(ctx, w: Tensor, ut: Tensor, qg: Tensor, mqk: Tensor, kr: Tensor, gc: Tensor) -> Tensor:  # noqa: ANN001
        if w.is_cuda:
            o, hs, us = native().gdn_fwd(w, ut, qg, mqk, kr, gc)
        else:
            o, hs, us = scan_reference(w, ut, qg, mqk, kr, gc)
        ctx.save_for_backward(w, qg, mqk, kr, gc, hs, us)
        return o

    @staticmethod
    def backward(ctx, do: Tensor) -> tuple[Tensor, ...]:  # noqa: ANN001
        w, qg, mqk, kr, gc, hs, us = ctx.saved_tensors
        if do.is_cuda:
            do = do.to(torch.bfloat16).contiguous()
            du, dhs = native().gdn_bwd(kr, mqk, do, qg, w, gc)
            op = torch.bfloat16  # batched GEMMs on bf16 operands, fp32 accumulation
        else:
            do = do.float()
            du, dhs = scan_reference_bwd(kr, mqk, do, qg, w, gc)
            op = torch.float32
        h, dhb, dub, u = hs.to(op), dhs.to(op), du.to(op), us.to(op)
        ht = h.transpose(-1, -2)
        dw = -(dub @ ht)                          # U = Ut - W H
        dqg = do.to(op) @ ht                      # O = Qg H + ...
        dmqk = do.to(op) @ u.transpose(-1, -2)    # ... + Mqk U
        dkr = u @ dhb.transpose(-1, -2)           # H' = gC H + Kr^T U
        dgc = (hs.float() * dhs.float()).sum((-1, -2))
        return dw.float(), du, dqg.float(), dmqk.float(), dkr.float(), dgc


def chunk_operands(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, *, l2norm: bool = True) -> tuple[Tensor, ...]:
    """The scan's chunk-parallel operands (W, Ut, Qg, Mqk, Kr, gC), fp32, ``[B*H, n, C, *]``.

    Inputs as for :func:`gated_delta_rule`; sequences are padded to whole chunks with zero
    keys / values, beta 0 and no decay, which leaves the state unchanged.
    """
    B, S, H, dk = k.shape
    dv = v.shape[-1]
    C = CHUNK
    q, k = q.float(), k.float()
    if l2norm:
        q, k = _l2n(q), _l2n(k)
    q = q / math.sqrt(dk)
    q, k, v = (x.float().transpose(1, 2) for x in (q, k, v))
    g, beta = g.float().transpose(1, 2), beta.float().transpose(1, 2)
    pad = (-S) % C
    if pad:
        q, k, v = (F.pad(x, (0, 0, 0, pad)) for x in (q, k, v))
        g, beta = F.pad(g, (0, pad)), F.pad(beta, (0, pad))
    n = (S + pad) // C
    q, k, v = (x.reshape(B * H, n, C, -1) for x in (q, k, v))
    g, beta = g.reshape(B * H, n, C), beta.reshape(B * H, n, C)

    G = g.cumsum(-1)
    lower = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    decay = torch.where(lower, G[..., :, None] - G[..., None, :], float("-inf")).exp()  # exp(G_t - G_s), s <= t
    a = (beta[..., :, None] * decay * (k @ k.transpose(-1, -2))).tril(-1)
    gam = G.exp()
    rhs = torch.cat([beta[..., None] * v, (beta * gam)[..., None] * k], -1)
    eye = torch.eye(C, device=q.device)
    sol = torch.linalg.solve_triangular(eye + a, rhs, upper=False, unitriangular=True)
    ut, w = sol[..., :dv], sol[..., dv:]
    mqk = decay * (q @ k.transpose(-1, -2))
    qg = gam[..., None] * q
    kr = (G[..., -1:] - G).exp()[..., None] * k
    gc = G[..., -1].exp()
    return w, ut, qg, mqk, kr, gc


def gated_delta_rule(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, *, l2norm: bool = True) -> Tensor:
    """``[B, S, H, dk]`` q / k, ``[B, S, H, dv]`` v, ``[B, S, H]`` log-decay g and beta -> ``[B, S, H, dv]``.

    q and k are L2-normalized over their head dim when ``l2norm`` (the reference's
    ``use_qk_l2norm_in_kernel``); q is scaled by ``dk ** -0.5``. Output in v's dtype.
    """
    B, S, H, _ = k.shape
    dv = v.shape[-1]
    w, ut, qg, mqk, kr, gc = chunk_operands(q, k, v, g, beta, l2norm=l2norm)
    n = w.shape[1]
    if w.is_cuda:
        op = torch.bfloat16
        o = _Scan.apply(w.to(op).contiguous(), ut.contiguous(), qg.to(op).contiguous(), mqk.to(op).contiguous(),
                        kr.to(op).contiguous(), gc.contiguous())  # fmt: skip
    else:
        o = _Scan.apply(w, ut, qg, mqk, kr, gc)
    o = o.reshape(B, H, n * CHUNK, dv)[:, :, :S].transpose(1, 2)
    return o.to(v.dtype)
