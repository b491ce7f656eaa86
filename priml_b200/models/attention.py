"""Attention blocks (``priml/model/attention.py:29-960``).

Layout everywhere is ``[..., S, heads, channels_head]``. ``SdpaFused`` runs the
hand-written sm_100a flash-attention kernel on CUDA (causal / sliding window,
grouped KV heads read in place -- no ``repeat_interleave``) and ATen SDPA on
CPU. ``SdpaNaive`` is matmul + fp32 softmax + matmul (HF eager order), used for
bit-parity tests and DTensor tensor parallelism.
"""

from __future__ import annotations

from dataclasses import KW_ONLY, field
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, HeadGeometry, RotaryFactors, propagate_attr
from priml_b200.models.init import InitFn, kaiming_uniform
from priml_b200.models.kvcache import KVCache
from priml_b200.models.linear import EnsembleLinear, Linear
from priml_b200.models.rope import RoPE

__all__ = [
    "MultiStreamAttention",
    "OutputGate",
    "SdpaFused",
    "SdpaNaive",
    "SelfAttention",
    "layer_window",
    "window_mask",
    "window_sizes",
]


_WINDOW_SHARE = {"S": 2, "L": 1}  # a short layer sees half the context, a long layer all of it


def layer_window(*, depth: int, max_seq_len: int, pattern: str) -> int:
    """Window of layer ``depth`` from a cycled ``S`` (half) / ``L`` (full) pattern."""
    letters = pattern.upper()
    unknown = sorted(set(letters) - set(_WINDOW_SHARE))
    if not letters or unknown:
        raise ValueError(f"window pattern {pattern!r} needs one or more letters from 'S' / 'L' (found {unknown}).")
    return max_seq_len // _WINDOW_SHARE[letters[depth % len(letters)]]


def window_sizes(*, num_layers: int, max_seq_len: int, pattern: str) -> list[int]:
    """Every layer's window; the last layer always sees the full context."""
    ws = [layer_window(depth=i, max_seq_len=max_seq_len, pattern=pattern) for i in range(num_layers)]
    ws[-1] = max_seq_len
    return ws


def window_mask(q: Tensor, k: Tensor, *, window: int) -> Tensor | None:
    """Additive causal mask admitting keys with ``0 <= q_pos - k_pos <= window``."""
    s, t = q.shape[-3], k.shape[-3]
    if window < 0 or window >= t:
        return None
    idx = torch.arange(t, device=q.device)
    offset = idx[t - s :, None] - idx[None, :]
    ok = (offset >= 0) & (offset <= window)
    return torch.zeros(s, t, dtype=q.dtype, device=q.device).masked_fill(~ok, float("-inf"))


def _expand_kv(q: Tensor, k: Tensor, v: Tensor) -> tuple[Tensor, Tensor]:
    g = q.shape[-2] // k.shape[-2]
    if g > 1:
        k = k.repeat_interleave(g, dim=-2)
        v = v.repeat_interleave(g, dim=-2)
    return k, v


class SdpaFused(nn.Module):
    """Fused attention. CUDA: the tcgen05 flash kernel (native GQA, causal,
    window). CPU or an explicit additive mask: ATen SDPA."""

    supports_gqa = True

    class Config(Fig["SdpaFused"]):
        pass

    def __init__(self, config: Config | None = None) -> None:
        del config
        super().__init__()

    def forward(
        self,
        q: Tensor,
        k: Tensor,
        v: Tensor,
        *,
        dropout_p: float = 0.0,
        is_causal: bool = False,
        attn_mask: Tensor | None = None,
        window: int = -1,
        **kwargs: Any,
    ) -> Tensor:
        del kwargs
        if attn_mask is None and dropout_p == 0.0 and q.ndim == 4 and ops.use_native(q):
            t = k.shape[-3]
            win = None if window < 0 or window >= t else window
            if is_causal or win is not None or q.shape[-3] == t:
                return ops.attention(q, k, v, causal=is_causal or win is not None, window=win)
        k, v = _expand_kv(q, k, v)
        if attn_mask is None:
            attn_mask = window_mask(q, k, window=window)
        qt, kt, vt = (x.movedim(-3, -2) for x in (q, k, v))
        out = F.scaled_dot_product_attention(
            qt, kt, vt, attn_mask=attn_mask, dropout_p=dropout_p, is_causal=is_causal and attn_mask is None
        )
        return out.movedim(-3, -2)


class SdpaNaive(nn.Module):
    """matmul -> fp32 softmax -> matmul (HF ``eager_attention_forward`` order)."""

    supports_gqa = True

    class Config(Fig["SdpaNaive"]):
        pass

    def __init__(self, config: Config | None = None) -> None:
        del config
        super().__init__()

    def forward(
        self,
        q: Tensor,
        k: Tensor,
        v: Tensor,
        *,
        dropout_p: float = 0.0,
        is_causal: bool = False,
        attn_mask: Tensor | None = None,
        window: int = -1,
        **kwargs: Any,
    ) -> Tensor:
        del kwargs
        if type(q).__name__ == "DTensor":
            # Tensor parallel (DTensor) path: plain masks replicate implicitly.
            from torch.distributed.tensor.experimental import implicit_replication

            with implicit_replication():
                return self._attend(q, k, v, dropout_p, is_causal, attn_mask, window)
        return self._attend(q, k, v, dropout_p, is_causal, attn_mask, window)

    @staticmethod
    def _attend(q: Tensor, k: Tensor, v: Tensor, dropout_p: float, is_causal: bool, attn_mask: Tensor | None,
                window: int) -> Tensor:  # fmt: skip
        k, v = _expand_kv(q, k, v)
        if attn_mask is None:
            attn_mask = window_mask(q, k, window=window)
        q, k, v = (x.movedim(-3, -2) for x in (q, k, v))
        a = torch.matmul(q, k.transpose(-2, -1)) * q.shape[-1] ** -0.5
        if is_causal:
            s, t = q.shape[-2], k.shape[-2]
            keep = torch.ones(s, t, dtype=torch.bool, device=q.device).tril(diagonal=t - s)
            a = a.masked_fill(~keep, float("-inf"))
        if attn_mask is not None:
            a = a + attn_mask
        a = a.softmax(dim=-1, dtype=torch.float32).to(q.dtype)
        if dropout_p > 0.0:
            a = F.dropout(a, p=dropout_p)
        return torch.matmul(a, v).movedim(-3, -2)


def _infer_head_dims(cfg: Any) -> None:
    """Fill the one unknown of ``(channels_in, heads, channels_head)``."""
    if cfg.channels_in == -1 and cfg.heads != -1 and cfg.channels_head != -1:
        cfg.channels_in = cfg.heads * cfg.channels_head
    if cfg.channels_head == -1 and cfg.channels_in != -1 and cfg.heads != -1:
        if cfg.channels_in % cfg.heads:
            raise ValueError(f"channels_in={cfg.channels_in} not divisible by heads={cfg.heads}.")
        cfg.channels_head = cfg.channels_in // cfg.heads
    if cfg.heads == -1 and cfg.channels_in != -1 and cfg.channels_head != -1:
        if cfg.channels_in % cfg.channels_head:
            raise ValueError(f"channels_in={cfg.channels_in} not divisible by channels_head={cfg.channels_head}.")
        cfg.heads = cfg.channels_in // cfg.channels_head
    if -1 in (cfg.channels_in, cfg.heads, cfg.channels_head):
        raise ValueError(
            f"Need two of channels_in={cfg.channels_in}, heads={cfg.heads}, channels_head={cfg.channels_head}."
        )


def _causal_chunk_mask(q: Tensor, k: Tensor) -> Tensor | None:
    """Bottom-right aligned causal mask for a chunk of ``S`` queries over ``T`` keys."""
    s, t = q.shape[-3], k.shape[-3]
    if s == t:
        return None
    ok = torch.ones(s, t, dtype=torch.bool, device=q.device).tril(diagonal=t - s)
    return torch.zeros(s, t, dtype=q.dtype, device=q.device).masked_fill(~ok, float("-inf"))


class SelfAttention(nn.Module):
    """Multi-head / grouped-query self-attention with a fused QKV projection.

    ``proj_qkv.weight`` is ``[heads + 2*kv_heads, channels_head, C]`` (each head
    its own ensemble member, so Muon orthogonalizes heads independently) and
    ``proj_out.weight`` is ``[C, heads*channels_head]`` -- the reference layout.
    """

    class Config(Fig["SelfAttention"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        heads: int = 8
        channels_head: int = -1
        num_heads_kv: int = -1
        """KV heads for GQA (-1 = heads)."""
        bias: bool = False
        dropout: float = 0.0
        causal: bool = False
        rope: Makeable[RotaryFactors] | None = None
        norm_qk: Makeable[nn.Module] | None = None
        share_qk_norm: bool = True
        norm_out: Makeable[nn.Module] | None = None
        split_qkv_projection: bool = False
        attn_kernel: Makeable[nn.Module] = field(default_factory=SdpaFused.Config)
        init_weight: InitFn = kaiming_uniform
        depth: int = -1
        window: int = -1
        """Sliding window (keys looked back over, self included); -1 = full."""

        @property
        def channels_out(self) -> int:
            return self.channels_in

        def finalize(self):  # noqa: ANN201
            _infer_head_dims(self)
            if self.num_heads_kv == -1:
                self.num_heads_kv = self.heads
            if isinstance(self.norm_qk, ChannelsIn) and self.norm_qk.channels_in == -1:
                self.norm_qk.channels_in = self.channels_head
            if isinstance(self.norm_out, ChannelsIn) and self.norm_out.channels_in == -1:
                self.norm_out.channels_in = self.heads * self.channels_head
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.heads % config.num_heads_kv:
            raise ValueError(f"heads={config.heads} must be divisible by num_heads_kv={config.num_heads_kv}.")
        self.heads = config.heads
        self.channels_head = config.channels_head
        self.num_heads_kv = config.num_heads_kv
        self.kv_groups = config.heads // config.num_heads_kv
        self.dropout = config.dropout
        self.causal = config.causal
        self.depth = config.depth
        self.window = config.window
        self.split_qkv_projection = config.split_qkv_projection
        c = config.channels_in
        self.proj_qkv = EnsembleLinear.Config(
            channels_in=c,
            channels_out=config.channels_head,
            num_ensemble=config.heads + 2 * config.num_heads_kv,
            bias=config.bias,
            depth=config.depth,
            init_weight=config.init_weight,
            shard="colwise",
        ).make()
        self.proj_out = Linear.Config(
            channels_in=config.heads * config.channels_head,
            channels_out=c,
            bias=config.bias,
            depth=config.depth,
            init_weight=config.init_weight,
            shard="rowwise",
        ).make()
        if config.norm_qk is None:
            self.norm_q: nn.Module | None = None
            self.norm_k: nn.Module | None = None
        elif config.share_qk_norm:
            shared = config.norm_qk.make()
            self.norm_q = shared
            self.norm_k = shared
        else:
            self.norm_q = config.norm_qk.make()
            self.norm_k = config.norm_qk.make()
        self.norm_out = config.norm_out.make() if config.norm_out else None
        self.rope = config.rope.make() if config.rope else None
        self.attn_kernel = config.attn_kernel.make()

    def assert_tensor_parallel_compatible(self) -> None:
        """DTensor tensor parallelism needs the decomposed kernel."""
        from torch.distributed.tensor import DTensor

        if isinstance(self.attn_kernel, SdpaFused) and isinstance(self.proj_qkv.weight, DTensor):
            raise RuntimeError(
                "DTensor tensor parallelism requires attn_kernel=SdpaNaive; the fused kernel "
                "runs on local head shards through priml_b200.parallel.tensor_parallel instead."
            )

    def reset_parameters(self) -> None:
        self.proj_qkv.reset_parameters()
        self.proj_out.reset_parameters()
        seen: nn.Module | None = None
        for norm in (self.norm_q, self.norm_k):
            if norm is not None and norm is not seen:
                if hasattr(norm, "reset_parameters"):
                    norm.reset_parameters()
                seen = norm
        if self.norm_out is not None and hasattr(self.norm_out, "reset_parameters"):
            self.norm_out.reset_parameters()

    def alloc_kv_cache(
        self,
        *,
        batch: int | tuple[int, ...],
        max_seq: int,
        device: torch.device | str | None = None,
        dtype: torch.dtype | None = None,
    ) -> KVCache:
        return KVCache.alloc(
            batch=batch,
            heads=self.num_heads_kv,
            max_seq=max_seq,
            channels_head=self.channels_head,
            device=device,
            dtype=dtype,
        )

    def forward(
        self,
        x: Tensor,
        *args: Any,
        positions: Tensor | list[Tensor] | None = None,
        cos_sin: tuple[Tensor, Tensor] | None = None,
        cache: KVCache | None = None,
        **kwargs: Any,
    ) -> tuple[Tensor, KVCache]:
        del args, kwargs
        s = x.shape[-2]
        if self.split_qkv_projection:
            q, k, v = self._split_qkv(x)
        else:
            q, k, v = self.proj_qkv(x).split([self.heads, self.num_heads_kv, self.num_heads_kv], dim=-2)
        if self.norm_q is not None:
            q = self.norm_q(q)
        if self.norm_k is not None:
            k = self.norm_k(k)
        if cos_sin is not None:
            q, k = RoPE.rotate(q, k, *cos_sin)
        elif self.rope is not None:
            if positions is None and cache is None and type(self.rope) is RoPE:
                cos, sin = self.rope.table(s, x.device)
            elif positions is None:
                offset = cache.seen if cache is not None else 0
                cos, sin = self.rope(torch.arange(offset, offset + s, device=x.device))
            else:
                assert isinstance(positions, Tensor)
                cos, sin = self.rope(positions)
            q, k = RoPE.rotate(q, k, cos, sin)

        attend = getattr(cache, "attend", None)
        if attend is not None:
            # a cache that attends itself (static buffers with device-side lengths)
            out = attend(q, k, v, window=self.window).flatten(-2)
            if self.norm_out is not None:
                out = self.norm_out(out)
            return self.proj_out(out), cache
        if cache is not None:
            kc, vc = cache.update(k.movedim(-3, -2), v.movedim(-3, -2))
            k, v = kc.movedim(-2, -3), vc.movedim(-2, -3)
        else:
            cache = KVCache(k.movedim(-3, -2), v.movedim(-3, -2))

        kernel = self.attn_kernel
        if not getattr(kernel, "supports_gqa", False):
            k, v = _expand_kv(q, k, v)
        t = k.shape[-3]
        causal_square = self.causal and t == s
        out = kernel(
            q,
            k,
            v,
            dropout_p=self.dropout if self.training else 0.0,
            is_causal=causal_square,
            attn_mask=_causal_chunk_mask(q, k) if self.causal and not causal_square else None,
            window=self.window,
        )
        out = out.flatten(-2)
        if self.norm_out is not None:
            out = self.norm_out(out)
        return self.proj_out(out), cache

    def _split_qkv(self, x: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        c = self.channels_head
        h, kv = self.heads, self.num_heads_kv
        w = self.proj_qkv.weight.to(x.dtype)
        b = None if self.proj_qkv.bias is None else self.proj_qkv.bias.to(x.dtype)
        parts = []
        for lo, hi in ((0, h), (h, h + kv), (h + kv, h + 2 * kv)):
            y = torch.matmul(x, w[lo:hi].reshape((hi - lo) * c, -1).T)
            if b is not None:
                y = y + b[lo:hi].reshape(-1)
            parts.append(y.reshape(*x.shape[:-1], hi - lo, c))
        return parts[0], parts[1], parts[2]


class OutputGate(nn.Module):
    """``inner(x) * sigmoid(gate_proj(x))``."""

    class Config(Fig["OutputGate"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        inner: Makeable[nn.Module] = field(default_factory=SelfAttention.Config)
        bias: bool = False
        depth: int = -1

        @property
        def channels_out(self) -> int:
            return self.channels_in

        @property
        def heads(self) -> int:
            return self.inner.heads if isinstance(self.inner, HeadGeometry) else 1

        @property
        def channels_head(self) -> int:
            return self.inner.channels_head if isinstance(self.inner, HeadGeometry) else self.channels_in

        def finalize(self):  # noqa: ANN201
            propagate_attr(self.inner, "channels_in", self.channels_in, protocol=ChannelsIn)
            propagate_attr(self.inner, "channels_out", self.channels_out, protocol=ChannelsOut)
            propagate_attr(self.inner, "depth", self.depth)
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.inner = config.inner.make()
        self.gate_proj = Linear.Config(
            channels_in=config.channels_in, channels_out=config.channels_in, bias=config.bias
        ).make()

    def reset_parameters(self) -> None:
        if hasattr(self.inner, "reset_parameters"):
            self.inner.reset_parameters()
        self.gate_proj.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Any:
        gate = torch.sigmoid(self.gate_proj(x))
        res = self.inner(x, *args, **kwargs)
        if isinstance(res, tuple):
            return res[0] * gate, res[1]
        return res * gate


class MultiStreamAttention(nn.Module):
    """Joint attention over N token streams (MMDiT style): each stream has its
    own QKV / output projections; attention runs over the concatenation of all
    streams' tokens (``priml/model/attention.py:532-869``)."""

    class Config(Fig["MultiStreamAttention"], kw_only=False):
        channels_in: int | list[int] = -1
        _: KW_ONLY
        num_streams: int = 2
        heads: int = 8
        channels_head: int = -1
        bias: bool = False
        norm_qk: Makeable[nn.Module] | None = None
        attn_kernel: Makeable[nn.Module] = field(default_factory=SdpaFused.Config)
        init_weight: InitFn = kaiming_uniform
        depth: int = -1

        def finalize(self):  # noqa: ANN201
            widths = self.channels_in if isinstance(self.channels_in, list) else [self.channels_in] * self.num_streams
            if len(widths) != self.num_streams:
                raise ValueError("channels_in list length must equal num_streams")
            if self.channels_head == -1:
                if widths[0] % self.heads:
                    raise ValueError("channels_in not divisible by heads")
                self.channels_head = widths[0] // self.heads
            if isinstance(self.norm_qk, ChannelsIn) and self.norm_qk.channels_in == -1:
                self.norm_qk.channels_in = self.channels_head
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        widths = config.channels_in if isinstance(config.channels_in, list) else [config.channels_in] * config.num_streams
        self.heads = config.heads
        self.channels_head = config.channels_head
        self.proj_qkvs = nn.ModuleList(
            EnsembleLinear.Config(
                channels_in=w,
                channels_out=config.channels_head,
                num_ensemble=3 * config.heads,
                bias=config.bias,
                depth=config.depth,
                init_weight=config.init_weight,
            ).make()
            for w in widths
        )
        self.proj_outs = nn.ModuleList(
            Linear.Config(
                channels_in=config.heads * config.channels_head,
                channels_out=w,
                bias=config.bias,
                depth=config.depth,
                init_weight=config.init_weight,
            ).make()
            for w in widths
        )
        # one q / k norm shared by every stream (the reference's state-dict layout)
        self.norm_q = config.norm_qk.make() if config.norm_qk else None
        self.norm_k = config.norm_qk.make() if config.norm_qk else None
        self.attn_kernel = config.attn_kernel.make()

    def reset_parameters(self) -> None:
        for m in (*self.proj_qkvs, *self.proj_outs):
            m.reset_parameters()

    def forward(self, streams: list[Tensor], *args: Any, **kwargs: Any) -> list[Tensor]:
        del args, kwargs
        qs, ks, vs, lens = [], [], [], []
        for i, x in enumerate(streams):
            q, k, v = self.proj_qkvs[i](x).split([self.heads] * 3, dim=-2)
            if self.norm_q is not None and self.norm_k is not None:
                q, k = self.norm_q(q), self.norm_k(k)
            qs.append(q)
            ks.append(k)
            vs.append(v)
            lens.append(x.shape[-2])
        out = self.attn_kernel(torch.cat(qs, -3), torch.cat(ks, -3), torch.cat(vs, -3))
        outs = out.flatten(-2).split(lens, dim=-2)
        return [self.proj_outs[i](o) for i, o in enumerate(outs)]
