"""Gated delta-rule linear attention (``priml/model/gated_delta_net.py:37-280``;
Yang, Kautz & Hatamizadeh 2024, "Gated Delta Networks").

Per value head, with state ``S`` (``[dv, dk]``), ``alpha_t = exp(g_t)`` and
``beta_t`` in (0, 1):

    S_t = alpha_t S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T,   o_t = S_t q_t

(q, k L2-normalized, q scaled by 1/sqrt(dk)). ``gated_delta_chunked`` evaluates
it in chunks of C tokens. Writing ``u_t = beta_t (v_t - alpha_t S_{t-1} k_t)``
the recurrence becomes ``S_t = alpha_t S_{t-1} + u_t k_t^T``; unrolled inside a
chunk from its entry state ``S0`` with ``gamma_t = prod_{r<=t} alpha_r``:

    (I + A) U = beta * (V - gamma * K S0^T),   A_ts = beta_t (gamma_t/gamma_s) k_s.k_t  (s < t)
    O   = gamma * Q S0^T + tril(gamma_t/gamma_s * Q K^T) U
    S_C = gamma_C S0 + (U * gamma_C/gamma)^T K

so each chunk costs one unit-lower-triangular solve and a few matmuls.
``gated_delta_recurrent`` is the token-by-token definition used as the oracle.
On CUDA with 128-wide heads the module runs ``priml_b200.ops.gated_delta``
(chunk-parallel algebra as batched GEMMs, the chunk scan on tcgen05 kernels).
"""

from __future__ import annotations

import math
from dataclasses import KW_ONLY, field
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsIn
from priml_b200.models.linear import Linear
from priml_b200.models.norm import CenteredRMSNorm
from priml_b200.ops import reference_forced
from priml_b200.ops.gated_delta import gated_delta_rule, kernel_supported

__all__ = ["GatedDeltaNet", "gated_delta_chunked", "gated_delta_recurrent"]


def _l2n(x: Tensor, eps: float = 1e-6) -> Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gated_delta_recurrent(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor) -> Tensor:
    """``[B, S, H, d]`` q/k/v, ``[B, S, H]`` g (log decay) and beta -> ``[B, S, H, dv]``."""
    B, S, H, dk = k.shape
    q = _l2n(q.float()) / math.sqrt(dk)
    k = _l2n(k.float())
    v, g, beta = v.float(), g.float(), beta.float()
    state = torch.zeros(B, H, v.shape[-1], dk, device=q.device)
    out = []
    for t in range(S):
        a = g[:, t].exp()[..., None, None]
        kt, vt, bt = k[:, t], v[:, t], beta[:, t][..., None]
        sk = torch.einsum("bhvk,bhk->bhv", state, kt)
        u = bt * (vt - a[..., 0] * sk)
        state = a * state + u[..., :, None] * kt[..., None, :]
        out.append(torch.einsum("bhvk,bhk->bhv", state, q[:, t]))
    return torch.stack(out, 1)


def gated_delta_chunked(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, chunk: int = 64) -> Tensor:
    B, S, H, dk = k.shape
    dv = v.shape[-1]
    dtype = v.dtype
    q = (_l2n(q.float()) / math.sqrt(dk)).transpose(1, 2)
    k = _l2n(k.float()).transpose(1, 2)
    v = v.float().transpose(1, 2)
    g = g.float().transpose(1, 2)
    beta = beta.float().transpose(1, 2)
    pad = (-S) % chunk
    if pad:
        q, k, v = (F.pad(x, (0, 0, 0, pad)) for x in (q, k, v))
        g, beta = F.pad(g, (0, pad)), F.pad(beta, (0, pad))
    n = (S + pad) // chunk
    q, k, v = (x.reshape(B, H, n, chunk, -1) for x in (q, k, v))
    g, beta = g.reshape(B, H, n, chunk), beta.reshape(B, H, n, chunk)
    G = g.cumsum(-1)
    eye = torch.eye(chunk, device=q.device)
    lower = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril()
    state = torch.zeros(B, H, dv, dk, device=q.device)
    out = torch.empty(B, H, n, chunk, dv, device=q.device)
    for c in range(n):
        qc, kc, vc, Gc, bc = q[:, :, c], k[:, :, c], v[:, :, c], G[:, :, c], beta[:, :, c]
        ratio = (Gc[..., :, None] - Gc[..., None, :]).masked_fill(~lower, float("-inf")).exp()  # gamma_t / gamma_s
        gam = Gc.exp()
        a = (bc[..., :, None] * ratio * (kc @ kc.transpose(-1, -2))).tril(-1)
        rhs = bc[..., None] * (vc - gam[..., None] * (kc @ state.transpose(-1, -2)))
        u = torch.linalg.solve_triangular(eye + a, rhs, upper=False, unitriangular=True)
        out[:, :, c] = gam[..., None] * (qc @ state.transpose(-1, -2)) + (ratio * (qc @ kc.transpose(-1, -2))) @ u
        to_end = (Gc[..., -1:] - Gc).exp()  # gamma_C / gamma_t in log space (gamma_t may underflow)
        state = gam[..., -1:, None] * state + (u * to_end[..., None]).transpose(-1, -2) @ kc
    out = out.reshape(B, H, n * chunk, dv)[:, :, :S]
    return out.transpose(1, 2).to(dtype)


class GatedDeltaNet(nn.Module):
    class Config(Fig["GatedDeltaNet"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        heads_k: int = 16
        heads_v: int = 32
        channels_k_head: int = 128
        channels_v_head: int = 128
        conv_kernel_size: int = 4
        norm: Makeable[nn.Module] = field(default_factory=CenteredRMSNorm.Config)
        depth: int = -1
        chunk_size: int = 64

        def finalize(self):  # noqa: ANN201
            if isinstance(self.norm, ChannelsIn) and self.norm.channels_in == -1:
                self.norm.channels_in = self.channels_v_head
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.heads_v % config.heads_k:
            raise ValueError(f"heads_v={config.heads_v} must be a multiple of heads_k={config.heads_k}.")
        h = config.channels_in
        self.heads_k, self.heads_v = config.heads_k, config.heads_v
        self.dk, self.dv = config.channels_k_head, config.channels_v_head
        self.chunk = config.chunk_size
        kd, vd = self.heads_k * self.dk, self.heads_v * self.dv
        conv = 2 * kd + vd
        self.in_proj_qkv = Linear.Config(h, conv).make()
        self.in_proj_z = Linear.Config(h, vd).make()
        self.in_proj_b = Linear.Config(h, self.heads_v).make()
        self.in_proj_a = Linear.Config(h, self.heads_v).make()
        self.conv1d = nn.Conv1d(conv, conv, config.conv_kernel_size, bias=False, groups=conv,
                                padding=config.conv_kernel_size - 1)  # fmt: skip
        self.dt_bias = nn.Parameter(torch.empty(self.heads_v))
        self.A_log = nn.Parameter(torch.empty(self.heads_v))
        self.norm = config.norm.make()
        self.out_proj = Linear.Config(vd, h).make()
        self.reset_parameters()

    def reset_parameters(self) -> None:
        for m in (self.in_proj_qkv, self.in_proj_z, self.in_proj_b, self.in_proj_a, self.conv1d, self.norm, self.out_proj):
            m.reset_parameters()
        with torch.no_grad():
            self.dt_bias.fill_(1.0)
            self.A_log.copy_(torch.empty_like(self.A_log).uniform_(0, 16).log())

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        shape = x.shape
        S = shape[-2]
        x = x.reshape(-1, S, shape[-1])
        kd, vd = self.heads_k * self.dk, self.heads_v * self.dv
        qkv = F.silu(self.conv1d(self.in_proj_qkv(x).transpose(1, 2))[:, :, :S]).transpose(1, 2)
        q, k, v = qkv.split([kd, kd, vd], dim=-1)
        z = self.in_proj_z(x).reshape(-1, S, self.heads_v, self.dv)
        beta = self.in_proj_b(x).sigmoid()
        g = -self.A_log.float().exp() * F.softplus(self.in_proj_a(x).float() + self.dt_bias)
        q = q.reshape(-1, S, self.heads_k, self.dk)
        k = k.reshape(-1, S, self.heads_k, self.dk)
        v = v.reshape(-1, S, self.heads_v, self.dv)
        r = self.heads_v // self.heads_k
        if r > 1:
            q, k = q.repeat_interleave(r, dim=-2), k.repeat_interleave(r, dim=-2)
        if x.is_cuda and kernel_supported(self.dk, self.dv) and not reference_forced():
            out = gated_delta_rule(q, k, v, g, beta)  # chunk scan on the tcgen05 kernels
        else:
            out = gated_delta_chunked(q, k, v, g, beta, chunk=self.chunk)
        out = self.norm(out.reshape(-1, self.dv)) * F.silu(z.reshape(-1, self.dv).float()).type_as(out)
        return self.out_proj(out.reshape(-1, S, vd)).reshape(*shape[:-1], -1)
