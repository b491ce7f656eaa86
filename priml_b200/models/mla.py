"""Multi-head latent attention, DeepSeek-V3 / Kimi-K2 style (``priml/model/mla.py:80-622``).

Per token the cache holds only the compressed latent ``c_kv`` (``kv_lora_rank``)
and the head-shared rotary key ``k_pe`` (``channels_qk_rope_head``).

Two mathematically equal evaluation orders are implemented:

* **absorbed** (decode, and the CPU oracle; the reference's only form):
  ``W_UK`` is folded into the query and attention runs in latent space -- K/V are
  never expanded. Cheapest when queries are few and the cache is long.
* **expanded** (training on CUDA): ``kv_b_proj`` expands the latent to per-head
  ``k_nope`` / ``v`` and the flash-attention kernel runs with
  ``D_qk = nope + rope`` and ``D_v`` -- for ``S == T`` this does
  ``(D_qk + D_v) / (L + R + L)`` of the absorbed form's attention FLOPs.
"""

from __future__ import annotations

from dataclasses import KW_ONLY, field
from functools import partial
from typing import Any, Literal

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, RotaryFactors
from priml_b200.models.init import InitFn, kaiming_uniform
from priml_b200.models.kvcache import KVCache
from priml_b200.models.linear import Linear
from priml_b200.models.norm import RMSNorm
from priml_b200.models.rope import RoPE

__all__ = ["MultiHeadLatentAttention"]


def _inherit(cfg: Any, **values: Any) -> None:
    """Give a projection's config the attention's settings wherever it still has its class default."""
    fields = type(cfg).__dataclass_fields__
    for name, value in values.items():
        if getattr(cfg, name) == fields[name].default:
            setattr(cfg, name, value)


class MultiHeadLatentAttention(nn.Module):
    class Config(Fig["MultiHeadLatentAttention"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        heads: int = -1
        channels_qk_nope_head: int = 128
        channels_qk_rope_head: int = 64
        channels_v_head: int = 128
        q_lora_rank: int | None = None
        kv_lora_rank: int = 512
        bias: bool = False
        dropout: float = 0.0
        causal: bool = True
        softmax_scale: float | None = None
        rope: Makeable[RotaryFactors] | None = None
        norm_q_lora: Makeable[nn.Module] = field(default_factory=partial(RMSNorm.Config, elementwise_affine=True))
        proj_q: Makeable[nn.Module] = field(default_factory=Linear.Config)
        proj_q_a: Makeable[nn.Module] = field(default_factory=Linear.Config)
        proj_q_b: Makeable[nn.Module] = field(default_factory=Linear.Config)
        proj_kv_a: Makeable[nn.Module] = field(default_factory=Linear.Config)
        proj_kv_b: Makeable[nn.Module] = field(default_factory=Linear.Config)
        proj_out: Makeable[nn.Module] = field(default_factory=Linear.Config)
        norm_kv_lora: Makeable[nn.Module] = field(default_factory=partial(RMSNorm.Config, elementwise_affine=True))
        init_weight: InitFn = kaiming_uniform
        depth: int = -1
        shard: Literal["colwise"] | None = None

        @property
        def channels_out(self) -> int:
            return self.channels_in

        @property
        def channels_qk_head(self) -> int:
            return self.channels_qk_nope_head + self.channels_qk_rope_head

        @property
        def channels_head(self) -> int:
            return self.channels_qk_head

        def finalize(self):  # noqa: ANN201
            if self.q_lora_rank is not None and isinstance(self.norm_q_lora, ChannelsIn) and self.norm_q_lora.channels_in == -1:
                self.norm_q_lora.channels_in = self.q_lora_rank
            if isinstance(self.norm_kv_lora, ChannelsIn) and self.norm_kv_lora.channels_in == -1:
                self.norm_kv_lora.channels_in = self.kv_lora_rank
            qk_out = self.heads * self.channels_qk_head
            slots: list[tuple[Any, int, int]] = [
                (self.proj_kv_a, self.channels_in, self.kv_lora_rank + self.channels_qk_rope_head),
                (self.proj_kv_b, self.kv_lora_rank, self.heads * (self.channels_qk_nope_head + self.channels_v_head)),
                (self.proj_out, self.heads * self.channels_v_head, self.channels_in),
            ]
            if self.q_lora_rank is None:
                slots.append((self.proj_q, self.channels_in, qk_out))
            else:
                slots.append((self.proj_q_a, self.channels_in, self.q_lora_rank))
                slots.append((self.proj_q_b, self.q_lora_rank, qk_out))
            for slot, c_in, c_out in slots:
                widths = {"channels_in": c_in, "channels_out": c_out}
                for attr, proto in (("channels_in", ChannelsIn), ("channels_out", ChannelsOut)):
                    if isinstance(slot, proto) and getattr(slot, attr) == -1:
                        setattr(slot, attr, widths[attr])
                if isinstance(slot, Linear.Config):
                    _inherit(slot, bias=self.bias, init_weight=self.init_weight)
                    slot.depth = self.depth if slot.depth == -1 else slot.depth
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.channels_in < 1:
            raise ValueError(f"channels_in must be > 0, got {config.channels_in}.")
        if config.heads < 1:
            raise ValueError(f"heads must be > 0, got {config.heads}.")
        if config.kv_lora_rank < 1:
            raise ValueError(f"kv_lora_rank must be > 0, got {config.kv_lora_rank}.")
        self.heads = config.heads
        self.channels_qk_nope_head = config.channels_qk_nope_head
        self.channels_qk_rope_head = config.channels_qk_rope_head
        self.channels_qk_head = config.channels_qk_nope_head + config.channels_qk_rope_head
        self.channels_v_head = config.channels_v_head
        self.q_lora_rank = config.q_lora_rank
        self.kv_lora_rank = config.kv_lora_rank
        self.dropout = config.dropout
        self.causal = config.causal
        self.depth = config.depth
        self.softmax_scale = self.channels_qk_head**-0.5 if config.softmax_scale is None else config.softmax_scale
        self.shard = config.shard
        self._tp_mesh: Any = None
        self._heads_local = config.heads
        self._head_offset = 0
        if config.q_lora_rank is None:
            self.q_proj: nn.Module | None = config.proj_q.make()
            self.q_a_proj: nn.Module | None = None
            self.q_a_layernorm: nn.Module | None = None
            self.q_b_proj: nn.Module | None = None
        else:
            self.q_proj = None
            self.q_a_proj = config.proj_q_a.make()
            self.q_a_layernorm = config.norm_q_lora.make()
            self.q_b_proj = config.proj_q_b.make()
        self.kv_a_proj = config.proj_kv_a.make()
        self.kv_a_layernorm = config.norm_kv_lora.make()
        self.kv_b_proj = config.proj_kv_b.make()
        self.o_proj = config.proj_out.make()
        self.rope = config.rope.make() if config.rope else None

    def reset_parameters(self) -> None:
        for m in (self.q_proj, self.q_a_proj, self.q_a_layernorm, self.q_b_proj, self.kv_a_proj,
                  self.kv_a_layernorm, self.kv_b_proj, self.o_proj):  # fmt: skip
            if m is not None and hasattr(m, "reset_parameters"):
                m.reset_parameters()

    def alloc_kv_cache(
        self,
        *,
        batch: int | tuple[int, ...],
        max_seq: int,
        device: torch.device | str | None = None,
        dtype: torch.dtype | None = None,
    ) -> KVCache:
        """Latent cache: ``k`` holds ``c_kv`` and ``v`` holds ``k_pe`` (one shared head)."""
        return KVCache.alloc(
            batch=batch,
            heads=1,
            max_seq=max_seq,
            channels_head=self.kv_lora_rank,
            channels_v_head=self.channels_qk_rope_head,
            device=device,
            dtype=dtype,
        )

    def _project_q(self, x: Tensor) -> Tensor:
        if self.q_proj is not None:
            q = self.q_proj(x)
        else:
            assert self.q_a_proj is not None and self.q_a_layernorm is not None and self.q_b_proj is not None
            q = self.q_b_proj(self.q_a_layernorm(self.q_a_proj(x)))
        return q.view(*q.shape[:-1], self._heads_local, self.channels_qk_head)

    def forward(
        self,
        x: Tensor,
        *args: Any,
        positions: Tensor | None = None,
        cos_sin: tuple[Tensor, Tensor] | None = None,
        cache: KVCache | None = None,
        **kwargs: Any,
    ) -> tuple[Tensor, KVCache]:
        del args, kwargs
        s = x.shape[-2]
        q = self._project_q(x)
        q_nope, q_pe = q[..., : self.channels_qk_nope_head], q[..., self.channels_qk_nope_head :]
        compressed = self.kv_a_proj(x)
        c_kv = self.kv_a_layernorm(compressed[..., : self.kv_lora_rank])
        k_pe = compressed[..., self.kv_lora_rank :].unsqueeze(-2)
        if cos_sin is None and self.rope is not None:
            if positions is None:
                offset = cache.seen if cache is not None else 0
                positions = torch.arange(offset, offset + s, device=x.device)
            cos_sin = self.rope(positions)
        if cos_sin is not None:
            q_pe, k_pe = RoPE.rotate(q_pe, k_pe, cos_sin[0], cos_sin[1], interleave=True)
        c_in, pe_in = c_kv.unsqueeze(-3), k_pe.movedim(-3, -2)
        if cache is not None:
            c_full, pe_full = cache.update(c_in, pe_in)
        else:
            cache = KVCache(c_in, pe_in)
            c_full, pe_full = c_in, pe_in
        c_full, pe_full = c_full.squeeze(-3), pe_full.squeeze(-3)
        t = c_full.shape[-2]
        if self._use_expanded(x, s, t):
            out = self._expanded_attention(q_nope, q_pe, c_full, pe_full)
        else:
            out = self._absorb_attention(q_nope, q_pe, c_full, pe_full, s, t)
        return self.o_proj(self._to_o_proj_input(out)), cache

    def _use_expanded(self, x: Tensor, s: int, t: int) -> bool:
        return s == t and s > 1 and ops.use_native(x) and self.training and self.dropout == 0.0

    def _w_kv_b(self) -> tuple[Tensor, Tensor]:
        rows = self.channels_qk_nope_head + self.channels_v_head
        lo = self._head_offset * rows
        w = self.kv_b_proj.weight[lo : lo + self._heads_local * rows].view(self._heads_local, rows, self.kv_lora_rank)
        return w[:, : self.channels_qk_nope_head, :], w[:, self.channels_qk_nope_head :, :]

    def _absorb_attention(self, q_nope: Tensor, q_pe: Tensor, c_kv: Tensor, k_pe: Tensor, s: int, t: int) -> Tensor:
        w_kr, w_uv = self._w_kv_b()
        w_kr, w_uv = w_kr.to(q_nope.dtype), w_uv.to(q_nope.dtype)
        q_abs = torch.einsum("...shd,hdl->...shl", q_nope, w_kr)
        if s == 1 and self._latent_decode_kernel(q_abs, q_pe, c_kv):
            # one new token per sequence: latent-space attention on the tcgen05 decode kernel
            lead = q_abs.shape[:-3]
            h = q_abs.shape[-2]
            q_cat = torch.cat([q_abs, q_pe.to(q_abs.dtype)], dim=-1).reshape(-1, h, q_abs.shape[-1] + q_pe.shape[-1])
            lat = ops.mla_decode(q_cat, c_kv.reshape(-1, t, c_kv.shape[-1]), k_pe.reshape(-1, t, k_pe.shape[-1]),
                                 scale=self.softmax_scale)  # fmt: skip
            lat = lat.view(*lead, 1, h, lat.shape[-1])
            return torch.einsum("...shl,hvl->...shv", lat, w_uv).flatten(-2)
        logits = torch.einsum("...shl,...tl->...hst", q_abs, c_kv) + torch.einsum("...shr,...tr->...hst", q_pe, k_pe)
        logits = logits * self.softmax_scale
        if self.causal and s > 1:
            logits = logits + torch.full((s, t), float("-inf"), device=logits.device, dtype=logits.dtype).triu(t - s + 1)
        attn = logits.softmax(dim=-1)
        if self.training and self.dropout > 0:
            attn = F.dropout(attn, p=self.dropout)
        lat = torch.einsum("...hst,...tl->...hsl", attn, c_kv)
        return torch.einsum("...hsl,hvl->...shv", lat, w_uv).flatten(-2)

    def _latent_decode_kernel(self, q_abs: Tensor, q_pe: Tensor, c_kv: Tensor) -> bool:
        """Whether a one-token step takes the decode kernel: CUDA bf16 inference with 512-wide
        latents and 64-wide rotary keys (the kernel's shapes)."""
        return (
            ops.use_native(q_abs)
            and not (torch.is_grad_enabled() and (q_abs.requires_grad or c_kv.requires_grad))
            and q_abs.dtype == torch.bfloat16
            and c_kv.dtype == torch.bfloat16
            and q_abs.shape[-1] == 512
            and q_pe.shape[-1] == 64
            and not (self.training and self.dropout > 0)
        )

    def _expanded_attention(self, q_nope: Tensor, q_pe: Tensor, c_kv: Tensor, k_pe: Tensor) -> Tensor:
        """Training order: expand K/V per head, then flash attention."""
        rows = self.channels_qk_nope_head + self.channels_v_head
        lo = self._head_offset * rows
        w = self.kv_b_proj.weight[lo : lo + self._heads_local * rows]
        kv = ops.linear(c_kv, w).view(*c_kv.shape[:-1], self._heads_local, rows)
        k_nope, v = kv[..., : self.channels_qk_nope_head], kv[..., self.channels_qk_nope_head :]
        k = torch.cat([k_nope, k_pe.unsqueeze(-2).expand(*k_nope.shape[:-1], self.channels_qk_rope_head)], dim=-1)
        q = torch.cat([q_nope, q_pe], dim=-1)
        out = ops.attention(q, k, v, causal=self.causal, scale=self.softmax_scale)
        return out.flatten(-2)

    def _to_o_proj_input(self, out: Tensor) -> Tensor:
        if self._tp_mesh is None:
            return out
        from torch.distributed.tensor import DTensor, Shard

        return DTensor.from_local(out, self._tp_mesh, [Shard(-1)], run_check=False)

    def shard_heads_over(self, mesh: Any) -> None:
        """Record this rank's head range for a head-parallel mesh."""
        tp = mesh.size()
        if self.heads % tp:
            raise ValueError(f"heads={self.heads} not divisible by tp={tp}.")
        self._tp_mesh = mesh
        self._heads_local = self.heads // tp
        self._head_offset = mesh.get_local_rank() * self._heads_local

    def tensor_parallel_plan(self) -> dict[str, Any]:
        from torch.distributed.tensor.parallel import ColwiseParallel, RowwiseParallel

        plan: dict[str, Any] = {"o_proj": RowwiseParallel()}
        if self.q_proj is not None:
            plan["q_proj"] = ColwiseParallel()
        else:
            plan["q_b_proj"] = ColwiseParallel()
        return plan

    def tensor_parallel_style(self) -> Any:
        """Head-parallel: q path and o_proj sharded over heads, latent replicated."""
        from priml_b200.parallel.tensor_parallel import MLAParallel

        return MLAParallel()
