"""Expert parallelism: MoE experts sharded over ranks, tokens exchanged over NVLink.

The reference has no expert parallelism (its MoE loops over all experts on
every rank, ``priml/model/moe.py:373-414``); this is the new capability for
MoE layers at scale. Each rank owns ``E / world`` experts (a contiguous slice of
the stacked expert weights) and keeps its own tokens (data parallel). Per MoE
layer:

1. route locally; all-gather the per-expert slot counts (``world x E`` ints,
   NCCL on a device tensor: no host synchronization);
2. build the plan on the device: every expert owner lays its rows out as
   128-aligned per-expert segments with the sources in rank order, so each
   source knows the destination row of each of its (token, choice) slots;
3. dispatch: every rank writes its slot rows straight into the owners' receive
   buffers (peer stores, ``ep.cu``), then the owner runs its experts as grouped
   tcgen05 GEMMs over the device-side segment offsets;
4. combine: the owner writes each output row back to its source's slot
   (peer stores), and the source forms ``sum_j w[t, j] y[t, j]``.

Backward runs the same two exchanges in the opposite directions. Without CUDA
(gloo ranks) an all-gather oracle implements the same exchange API.

Gradients follow the sequence-parallel TP strategy: replicated parameters are
averaged over all ranks once per step; expert weights (which saw the tokens of
every rank) are divided by the world size; the clip norm sums the expert
gradients' squares over the expert-parallel group.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor, nn

from priml_b200.config import Fig
from priml_b200.parallel.runtime import global_device_mesh
from priml_b200.parallel.strategies import place

__all__ = ["EpComm", "EpOracleComm", "EpPlan", "ExpertParallel", "ep_plan", "shard_experts"]

log = logging.getLogger(__name__)


@dataclass
class EpPlan:
    """Device-side dispatch plan of one MoE call on one rank."""

    tokens: int
    top_k: int
    dest_rank: Tensor  # int32 [S]: owner of each (token, choice) slot
    dest_row: Tensor  # int64 [S]: row in the owner's receive buffer
    meta: Tensor  # int32 [S]: (rank << 24) | slot, stored beside each row for the way back
    seg_start: Tensor  # int32 [EL + 1]: this rank's expert segments (grouped GEMM offsets)
    totals: Tensor  # int32 [EL]: real rows per local expert (the rest of a segment is padding)
    cap: int  # receive capacity (static bound)
    origin: Tensor | None = None  # int32 [cap]: (source rank << 24) | slot per received row, -1 = none

    @property
    def slots(self) -> int:
        return self.tokens * self.top_k


def _all_gather(t: Tensor, group: Any, world: int) -> Tensor:
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.stack(parts)


def ep_plan(indices: Tensor, num_experts: int, rank: int, world: int, group: Any = None) -> EpPlan:
    """Plan for ``[T, k]`` global expert indices; every rank must call it (one small all-gather)."""
    t, k = indices.shape
    flat = indices.reshape(-1).long()
    s = flat.numel()
    el = num_experts // world
    counts = torch.bincount(flat, minlength=num_experts)
    counts_all = _all_gather(counts, group, world) if world > 1 else counts.unsqueeze(0)  # [W, E]
    tot = counts_all.sum(0)
    padded = ((tot + 127) // 128 * 128).view(world, el)
    seg = padded.cumsum(1) - padded  # [W, EL] segment starts on each owner
    src_off = (counts_all.cumsum(0) - counts_all)[rank]  # [E] rows of lower ranks before ours
    order = torch.argsort(flat, stable=True)
    starts = torch.cumsum(counts, 0) - counts
    within = torch.empty_like(flat)
    within[order] = torch.arange(s, device=flat.device) - starts[flat[order]]
    dest_row = seg.reshape(-1)[flat] + src_off[flat] + within
    mine = torch.cat([seg[rank], (seg[rank, -1] + padded[rank, -1]).reshape(1)]).to(torch.int32)
    meta = (rank << 24) | torch.arange(s, device=flat.device, dtype=torch.int32)
    cap = (world * s + 127) // 128 * 128 + 128 * el
    return EpPlan(t, k, (flat // el).to(torch.int32), dest_row, meta, mine, tot.view(world, el)[rank].to(torch.int32), cap)


# --------------------------------------------------------------------------- communicators
class EpComm:
    """Row exchange over NVLink peer memory (native ``EpGroup``; buffers grow on demand,
    collectively: every rank makes the same calls with the same capacities)."""

    fused = True

    def __init__(self, group: Any, timeout_s: float = 60.0) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = timeout_s
        self._g: Any = None
        self._cap = (0, 0, 0)

    def _ensure(self, recv: int, back: int, cols: int) -> Any:
        if self._g is not None and recv <= self._cap[0] and back <= self._cap[1] and cols == self._cap[2]:
            return self._g
        from priml_b200.ops import native

        want = (max(recv, self._cap[0]), max(back, self._cap[1]), cols)
        # Every rank must size (and later fill) its buffers alike: the plan assumes equal token counts.
        seen: list[Any] = [None] * self.world
        dist.all_gather_object(seen, want, group=self.group)
        if any(s != want for s in seen):
            raise ValueError(f"expert parallelism needs the same tokens per MoE call on every rank; got {seen}")
        if self._g is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        g = native().EpGroup(self.rank, self.world, want[0], want[1], cols, self.timeout_s)
        handles: list[Any] = [None] * self.world
        dist.all_gather_object(handles, g.handles(), group=self.group)
        g.open(handles)
        self._g, self._cap = g, want
        return g

    def to_experts(self, src: Tensor, gather: Tensor | None, plan: EpPlan, with_meta: bool) -> tuple[Tensor, Tensor | None]:
        cols = src.shape[1]
        g = self._ensure(plan.cap, plan.slots, cols)
        g.scatter(0, src, gather, plan.dest_rank, plan.dest_row, plan.meta if with_meta else None)
        g.wait(0)
        priv = torch.empty(plan.cap, cols, device=src.device, dtype=torch.bfloat16)
        meta = torch.full((plan.cap,), -1, device=src.device, dtype=torch.int32) if with_meta else None
        g.collect(0, priv, meta, plan.seg_start, plan.totals)
        g.release(0)
        return priv, meta

    def to_sources(self, src: Tensor, origin: Tensor, plan: EpPlan) -> Tensor:
        cols = src.shape[1]
        g = self._ensure(plan.cap, plan.slots, cols)
        dest_rank = torch.where(origin >= 0, origin >> 24, -1).to(torch.int32)
        dest_row = (origin & 0xFFFFFF).long()
        g.scatter(1, src, None, dest_rank, dest_row, None)
        g.wait(1)
        out = g.rows(1)[: plan.slots].clone()
        g.release(1)
        return out


class EpOracleComm:
    """All-gather reference of :class:`EpComm` (any backend, any device)."""

    fused = False

    def __init__(self, group: Any, timeout_s: float = 60.0) -> None:
        del timeout_s
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def to_experts(self, src: Tensor, gather: Tensor | None, plan: EpPlan, with_meta: bool) -> tuple[Tensor, Tensor | None]:
        rows = src.index_select(0, gather) if gather is not None else src[: plan.slots]
        w = self.world
        rows_all = _all_gather(rows, self.group, w).reshape(-1, rows.shape[1])
        dr_all = _all_gather(plan.dest_rank, self.group, w).reshape(-1)
        row_all = _all_gather(plan.dest_row, self.group, w).reshape(-1)
        meta_all = _all_gather(plan.meta, self.group, w).reshape(-1)
        mask = dr_all == self.rank
        priv = torch.zeros(plan.cap, rows.shape[1], device=src.device, dtype=src.dtype)
        priv[row_all[mask]] = rows_all[mask]
        meta = None
        if with_meta:
            meta = torch.full((plan.cap,), -1, device=src.device, dtype=torch.int32)
            meta[row_all[mask]] = meta_all[mask]
        return priv, meta

    def to_sources(self, src: Tensor, origin: Tensor, plan: EpPlan) -> Tensor:
        w = self.world
        rows_all = _all_gather(src.contiguous(), self.group, w).reshape(-1, src.shape[1])
        org_all = _all_gather(origin, self.group, w).reshape(-1)
        mask = (org_all >= 0) & ((org_all >> 24) == self.rank)
        out = torch.zeros(plan.slots, src.shape[1], device=src.device, dtype=src.dtype)
        out[(org_all[mask] & 0xFFFFFF).long()] = rows_all[mask]
        return out


# --------------------------------------------------------------------------- autograd
class _ToExperts(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, plan: EpPlan, comm: Any) -> Tensor:  # type: ignore[override]
        tok = torch.arange(plan.tokens, device=x.device).repeat_interleave(plan.top_k)
        priv, meta = comm.to_experts(x, tok, plan, True)
        plan.origin = meta
        ctx.plan, ctx.comm, ctx.dtype = plan, comm, x.dtype
        return priv

    @staticmethod
    def backward(ctx, dpriv: Tensor):  # type: ignore[override]
        plan, comm = ctx.plan, ctx.comm
        d = dpriv.to(torch.bfloat16).contiguous() if comm.fused else dpriv.contiguous()
        slots = comm.to_sources(d, plan.origin, plan)
        dx = slots.float().view(plan.tokens, plan.top_k, -1).sum(1).to(ctx.dtype)
        return dx, None, None


class _ToSources(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y_priv: Tensor, plan: EpPlan, comm: Any) -> Tensor:  # type: ignore[override]
        ctx.plan, ctx.comm = plan, comm
        return comm.to_sources(y_priv.contiguous(), plan.origin, plan)

    @staticmethod
    def backward(ctx, dslots: Tensor):  # type: ignore[override]
        plan, comm = ctx.plan, ctx.comm
        d = dslots.to(torch.bfloat16).contiguous() if comm.fused else dslots.contiguous()
        priv, _ = comm.to_experts(d, None, plan, False)
        return priv, None, None


class EpDispatcher:
    """Installed on ``MoE.expert_parallel``: routes one MoE call through the owners' experts."""

    def __init__(self, comm: Any) -> None:
        self.comm = comm

    def __call__(self, moe: nn.Module, xf: Tensor, weights: Tensor, indices: Tensor) -> Tensor:
        from priml_b200 import ops

        comm = self.comm
        plan = ep_plan(indices, moe.num_experts, comm.rank, comm.world, comm.group)
        x = xf.to(torch.bfloat16) if comm.fused else xf
        x_priv = _ToExperts.apply(x, plan, comm)
        experts = moe.experts
        y_priv = ops.grouped_swiglu_mlp(x_priv, experts.up_proj, experts.down_proj, plan.seg_start)
        y_slots = _ToSources.apply(y_priv.to(x_priv.dtype), plan, comm)
        y = y_slots.float() * weights.reshape(-1, 1).float()
        return y.view(plan.tokens, plan.top_k, -1).sum(1).to(xf.dtype)


def shard_experts(model: nn.Module, comm: Any) -> list[nn.Parameter]:
    """Keep this rank's slice of every MoE's stacked experts and install the dispatcher."""
    from priml_b200.models.moe import GroupedSwiGLUExperts, MoE

    sharded: list[nn.Parameter] = []
    w, r = comm.world, comm.rank
    for mod in model.modules():
        if not isinstance(mod, MoE):
            continue
        ex = mod.experts
        if not isinstance(ex, GroupedSwiGLUExperts):
            raise NotImplementedError("expert parallelism needs stacked SwiGLU experts (GroupedSwiGLUExperts)")
        if mod.num_experts % w:
            raise ValueError(f"{mod.num_experts} experts do not divide over {w} ranks")
        el = mod.num_experts // w
        ex.up_proj = nn.Parameter(ex.up_proj.data[r * el : (r + 1) * el].clone())
        ex.down_proj = nn.Parameter(ex.down_proj.data[r * el : (r + 1) * el].clone())
        ex.num_experts = el
        ex.expert_offset = r * el
        mod.expert_parallel = EpDispatcher(comm)
        sharded += [ex.up_proj, ex.down_proj]
    return sharded


class ExpertParallel:
    """Strategy: experts sharded over the ``ep`` mesh axis (usually the data-parallel
    axis itself), every other parameter replicated with averaged gradients."""

    class Config(Fig["ExpertParallel"]):
        mesh_dim: str = "dp"
        timeout_s: float = 60.0
        comm: str = "auto"
        """``fused`` (NVLink kernels; CUDA), ``oracle`` (all-gather), ``auto`` = fused on CUDA."""

    def __init__(self, config: Config | None = None) -> None:
        from priml_b200.parallel.tp_fused import TpGradSync  # noqa: F401  (same gradient rules)

        config = config or ExpertParallel.Config()
        mesh = global_device_mesh()
        if mesh is None:
            raise RuntimeError("ExpertParallel requires the MultiProcess runtime.")
        names = mesh.mesh_dim_names or ()
        if config.mesh_dim not in names:
            raise ValueError(f"Mesh dimension {config.mesh_dim!r} not in {names}.")
        if len(names) > 1 and mesh.size() != mesh[config.mesh_dim].size():
            raise NotImplementedError("expert parallelism composes with a one-axis mesh only")
        self.group = mesh[config.mesh_dim].get_group()
        use_cuda = mesh.device_type == "cuda"
        self.device = torch.device("cuda", torch.cuda.current_device()) if use_cuda else torch.device(mesh.device_type)
        if config.comm not in ("auto", "fused", "oracle"):
            raise ValueError(f"comm must be auto, fused or oracle; got {config.comm!r}")
        if config.comm == "fused" and not use_cuda:
            raise RuntimeError("the fused expert exchange needs CUDA ranks")
        cls = EpComm if (use_cuda and config.comm != "oracle") else EpOracleComm
        self.comm = cls(self.group, config.timeout_s)
        self.sync: Any = None

    def __call__(self, model: nn.Module) -> nn.Module:
        from priml_b200.parallel.tp_fused import TpGradSync

        model = place(model, self.device)
        sharded = shard_experts(model, self.comm)
        model.to(self.device)
        self.sync = TpGradSync(model, sharded, None, dist.get_world_size())
        log.info("Expert parallelism over %d ranks: %d expert weights sharded.", self.comm.world, len(sharded))
        return model

    def build_optimizer(self, make: Any, model: nn.Module) -> Any:
        from priml_b200.parallel.tp_fused import TpOptimizer

        assert self.sync is not None, "apply the strategy to the model first"
        base = make([p for p in model.parameters() if p.requires_grad])
        return TpOptimizer(base, self.sync, self.group)
