"""Token router and mixture-of-experts FFN (``priml/model/moe.py:79-442``).

Routing matches the reference: softmax (Switch, with the load-balance aux loss)
or sigmoid with the aux-loss-free ``e_score_correction_bias`` (DeepSeek-V3), optional
grouped top-k, renormalization and ``routed_scaling_factor``.

Dispatch is different by design. The reference loops over active experts in
Python after a ``.tolist()`` host sync. Here the routed SwiGLU experts are held
**stacked** -- ``experts.up_proj [E, 2H, C]`` and ``experts.down_proj [E, C, H]`` --
so that

* on CUDA, tokens are permuted by expert on the device and both expert GEMMs
  run as single grouped tcgen05 GEMMs over device-side group offsets (no host
  sync), and
* expert parallelism shards the leading ``E`` axis (``priml_b200.parallel.expert``).

``state_dict`` / ``load_state_dict`` still speak the reference's per-expert keys
(``experts.{e}.up_proj.weight``, ``experts.{e}.down_proj.weight``), so
checkpoints interchange.
"""

from __future__ import annotations

import math
from dataclasses import KW_ONLY, field
from typing import Any, Literal

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from priml_b200 import ops
from priml_b200.config import Fig, Makeable
from priml_b200.models.custom_types import ChannelsIn, ChannelsOut, ShardableConfig, propagate_attr
from priml_b200.models.swiglu import SwiGLU

__all__ = ["GroupedSwiGLUExperts", "MoE", "Router", "moe_dispatch_plan"]


class Router(nn.Module):
    """Top-k router returning ``(weights [T,k], indices [T,k], logits [T,E])``."""

    class Config(Fig["Router"], kw_only=False):
        channels_in: int = -1
        _: KW_ONLY
        num_experts: int = 8
        top_k: int = 2
        jitter_noise: float = 0.0
        scoring_func: Literal["softmax", "sigmoid"] = "softmax"
        norm_topk_prob: bool | None = None
        routed_scaling_factor: float = 1.0
        n_group: int = 1
        topk_group: int = 1
        use_correction_bias: bool | None = None

        def finalize(self):  # noqa: ANN201
            sigmoid = self.scoring_func == "sigmoid"
            if self.norm_topk_prob is None:
                self.norm_topk_prob = sigmoid
            if self.use_correction_bias is None:
                self.use_correction_bias = sigmoid
            if self.num_experts % self.n_group:
                raise ValueError(f"num_experts={self.num_experts} must be divisible by n_group={self.n_group}.")
            if self.topk_group > self.n_group:
                raise ValueError(f"topk_group={self.topk_group} > n_group={self.n_group}.")
            if not 1 <= self.top_k <= self.num_experts:
                raise ValueError(f"top_k={self.top_k} must satisfy 1 <= top_k <= num_experts={self.num_experts}.")
            if self.n_group > 1 and self.top_k > self.topk_group * (self.num_experts // self.n_group):
                raise ValueError("top_k exceeds the experts eligible after grouped routing.")
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        if config.scoring_func not in ("softmax", "sigmoid"):
            raise ValueError(f"scoring_func={config.scoring_func!r} must be 'softmax' or 'sigmoid'.")
        self.num_experts = config.num_experts
        self.top_k = config.top_k
        self.jitter_noise = config.jitter_noise
        self.scoring_func = config.scoring_func
        self.norm_topk_prob = bool(config.norm_topk_prob)
        self.routed_scaling_factor = config.routed_scaling_factor
        self.n_group = config.n_group
        self.topk_group = config.topk_group
        self.gate = nn.Linear(config.channels_in, config.num_experts, bias=False)
        if config.use_correction_bias:
            self.register_buffer("e_score_correction_bias", torch.zeros(config.num_experts))
        else:
            self.e_score_correction_bias = None

    def reset_parameters(self) -> None:
        nn.init.kaiming_uniform_(self.gate.weight, a=math.sqrt(5))
        if self.e_score_correction_bias is not None:
            self.e_score_correction_bias.zero_()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> tuple[Tensor, Tensor, Tensor]:
        del args, kwargs
        if self.training and self.jitter_noise > 0:
            x = x * torch.empty_like(x).uniform_(1 - self.jitter_noise, 1 + self.jitter_noise)
        logits = ops.linear(x, self.gate.weight).float()
        scores = logits.sigmoid() if self.scoring_func == "sigmoid" else logits.softmax(dim=-1)
        sel = scores + self.e_score_correction_bias if self.e_score_correction_bias is not None else scores
        if self.n_group > 1:
            sel = self._mask_inactive_groups(sel)
        _, indices = sel.topk(self.top_k, dim=-1)
        weights = scores.gather(-1, indices)
        if self.norm_topk_prob:
            weights = weights / weights.sum(dim=-1, keepdim=True).clamp(min=1e-20)
        return weights * self.routed_scaling_factor, indices, logits

    def _mask_inactive_groups(self, sel: Tensor) -> Tensor:
        t = sel.shape[0]
        gs = self.num_experts // self.n_group
        grouped = sel.view(t, self.n_group, gs)
        group_scores = grouped.topk(min(2, gs), dim=-1).values.sum(dim=-1)
        top = group_scores.topk(self.topk_group, dim=-1).indices
        keep = torch.zeros_like(group_scores, dtype=torch.bool).scatter_(1, top, True)
        return sel.masked_fill(~keep.unsqueeze(-1).expand(-1, -1, gs).reshape(t, -1), float("-inf"))


def moe_dispatch_plan(indices: Tensor, num_experts: int) -> tuple[Tensor, Tensor, Tensor]:
    """Device-side dispatch plan for ``[T, k]`` expert indices.

    Returns ``(order, token_of_slot, offsets)``: ``order`` sorts the ``T*k``
    (token, choice) slots by expert (stable), ``token_of_slot`` is the source
    token of each sorted slot, and ``offsets [E+1]`` delimits each expert's rows.
    No host synchronization.
    """
    t, k = indices.shape
    flat = indices.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=num_experts)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64, device=indices.device)
    offsets[1:] = torch.cumsum(counts, 0)
    token_of_slot = torch.div(order, k, rounding_mode="floor")
    return order, token_of_slot, offsets


class GroupedSwiGLUExperts(nn.Module):
    """``E`` SwiGLU experts stored stacked: ``up_proj [E, 2H, C]`` (gate rows
    first within each expert) and ``down_proj [E, C, H]``."""

    def __init__(self, num_experts: int, channels_in: int, channels_hidden: int, channels_out: int, template: SwiGLU) -> None:
        super().__init__()
        self.num_experts = num_experts
        self.channels_hidden = channels_hidden
        self.up_proj = nn.Parameter(torch.empty(num_experts, 2 * channels_hidden, channels_in))
        self.down_proj = nn.Parameter(torch.empty(num_experts, channels_out, channels_hidden))
        self._template = [template]  # init functions only; not a submodule
        self.reset_parameters()

    def reset_parameters(self) -> None:
        tpl = self._template[0]
        if tpl.up_proj.weight.device != self.up_proj.device:  # built on meta, materialized since
            tpl.to_empty(device=self.up_proj.device)
        with torch.no_grad():
            for e in range(self.num_experts):
                tpl.reset_parameters()
                self.up_proj[e].copy_(tpl.up_proj.weight)
                self.down_proj[e].copy_(tpl.down_proj.weight)

    def forward(self, x_sorted: Tensor, offsets: Tensor) -> Tensor:
        """Rows ``offsets[e]:offsets[e+1]`` of ``x_sorted`` go through expert ``e`` (on CUDA the
        segments start on multiples of 128: ``priml_b200.ops.grouped.padded_dispatch_plan``)."""
        return ops.grouped_swiglu_mlp(x_sorted, self.up_proj, self.down_proj, offsets)


class MoE(nn.Module):
    """Routed experts plus always-on shared experts."""

    class Config(Fig["MoE"], kw_only=False):
        channels_in: int = -1
        channels_out: int = -1
        _: KW_ONLY
        router: Any = field(default_factory=Router.Config)
        expert: Makeable[nn.Module] = field(default_factory=SwiGLU.Config)
        num_shared_experts: int = 0
        shared_expert: Makeable[nn.Module] = field(default_factory=SwiGLU.Config)
        aux_loss_weight: float = 0.01
        depth: int = -1

        def finalize(self):  # noqa: ANN201
            if self.channels_in == -1:
                self.channels_in = self.channels_out
            if self.channels_out == -1:
                self.channels_out = self.channels_in
            self.router.channels_in = self.channels_in
            for cfg in (self.expert, self.shared_expert):
                propagate_attr(cfg, "channels_in", self.channels_in, protocol=ChannelsIn)
                propagate_attr(cfg, "channels_out", self.channels_out, protocol=ChannelsOut)
                propagate_attr(cfg, "depth", self.depth)
                if isinstance(cfg, ShardableConfig):
                    cfg.shard = "colwise"
            return super().finalize()

    def __init__(self, config: Config) -> None:
        super().__init__()
        self.num_experts = config.router.num_experts
        self.top_k = config.router.top_k
        self.channels_out = config.channels_out
        self.aux_loss_weight = config.aux_loss_weight
        self.depth = config.depth
        self.router = config.router.make()
        template = config.expert.make()
        self._grouped = (
            isinstance(template, SwiGLU)
            and type(template) is SwiGLU
            and template.gate
            and template.norm is None
            and template.act is F.silu
            and template.up_proj.bias is None
        )
        if self._grouped:
            self.experts: nn.Module = GroupedSwiGLUExperts(
                self.num_experts, config.channels_in, template.channels_hidden, config.channels_out, template
            )
            self._register_state_dict_hook(_split_expert_keys)
            self._register_load_state_dict_pre_hook(_stack_expert_keys, with_module=True)
        else:
            self.experts = nn.ModuleList([template] + [config.expert.make() for _ in range(self.num_experts - 1)])
        self.shared_experts = nn.ModuleList([config.shared_expert.make() for _ in range(config.num_shared_experts)])
        self.register_buffer("_aux_loss", torch.tensor(0.0), persistent=False)
        # Expert parallelism installs a dispatcher here (priml_b200.parallel.expert).
        self.expert_parallel: Any = None

    @property
    def aux_loss(self) -> Tensor:
        return self._aux_loss

    def reset_parameters(self) -> None:
        self._aux_loss.zero_()
        self.router.reset_parameters()
        if isinstance(self.experts, GroupedSwiGLUExperts):
            self.experts.reset_parameters()
        else:
            for e in self.experts:
                e.reset_parameters()
        for s in self.shared_experts:
            s.reset_parameters()

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        weights, indices, logits = self.router(xf)
        if self.training and self.aux_loss_weight > 0 and self.router.scoring_func == "softmax":
            self._aux_loss = self._load_balance_loss(logits, indices)
        if self.expert_parallel is not None:
            y = self.expert_parallel(self, xf, weights, indices)
        elif self._grouped:
            y = self._dispatch_grouped(xf, weights, indices)
        else:
            y = self._dispatch_loop(xf, weights, indices)
        for shared in self.shared_experts:
            y = y + shared(xf)
        return y.reshape(*shape[:-1], self.channels_out)

    def _dispatch_grouped(self, xf: Tensor, weights: Tensor, indices: Tensor) -> Tensor:
        # padded device-side dispatch -> grouped expert GEMMs -> weighted combine (no host sync)
        return ops.grouped_swiglu_experts(xf, weights, indices, self.experts.up_proj, self.experts.down_proj)

    def _dispatch_loop(self, xf: Tensor, weights: Tensor, indices: Tensor) -> Tensor:
        order, tok, offsets = moe_dispatch_plan(indices, self.num_experts)
        w_sorted = weights.reshape(-1)[order].unsqueeze(-1)
        y = xf.new_zeros(xf.shape[0], self.channels_out)
        bounds = offsets.tolist()
        for e in range(self.num_experts):
            lo, hi = bounds[e], bounds[e + 1]
            if hi > lo:
                t = tok[lo:hi]
                y.index_add_(0, t, (self.experts[e](xf.index_select(0, t)) * w_sorted[lo:hi]).to(y.dtype))
        return y

    def _load_balance_loss(self, logits: Tensor, indices: Tensor) -> Tensor:
        """Switch Transformer loss ``E * sum_e f_e * P_e * weight``."""
        t = logits.shape[0]
        probs = logits.softmax(dim=-1)
        counts = torch.zeros(self.num_experts, device=logits.device, dtype=logits.dtype)
        counts.scatter_add_(0, indices.reshape(-1), torch.ones(indices.numel(), device=logits.device, dtype=logits.dtype))
        freq = counts / (t * self.top_k)
        return self.num_experts * (freq * probs.mean(dim=0)).sum() * self.aux_loss_weight


def _split_expert_keys(module: nn.Module, state: dict[str, Any], prefix: str, local_metadata: Any) -> None:
    del local_metadata
    base = getattr(module.experts, "expert_offset", 0)  # expert parallelism: this rank's first global expert
    for name in ("up_proj", "down_proj"):
        key = f"{prefix}experts.{name}"
        if key in state:
            stacked = state.pop(key)
            for e in range(stacked.shape[0]):
                state[f"{prefix}experts.{base + e}.{name}.weight"] = stacked[e]


def _stack_expert_keys(module: nn.Module, state: dict[str, Any], prefix: str, *args: Any) -> None:
    del args
    ex = module.experts  # type: ignore[attr-defined]
    base = getattr(ex, "expert_offset", 0)
    n = ex.num_experts
    for name in ("up_proj", "down_proj"):
        keys = [f"{prefix}experts.{base + e}.{name}.weight" for e in range(n)]
        if all(k in state for k in keys):
            state[f"{prefix}experts.{name}"] = torch.stack([state.pop(k) for k in keys])
