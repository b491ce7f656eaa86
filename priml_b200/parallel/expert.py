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

With ``comm="gemm"`` (the default on CUDA) the exchange happens inside the
expert GEMMs (``ops/csrc/ep_gemm.cu``): the up projection's copy warps pull
every received row from its source's send buffer over NVLink while the tensor
cores run the chunks already in place, and the down projection's epilogue
stores each output row straight into its source's receive buffer. Backward
mirrors it (the down dgrad pulls ``w * dy``, the up dgrad pushes ``dx``). The
plan then all-gathers the routing indices instead of the counts, so every
owner knows the source of each row it receives.

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

__all__ = [
    "EpComm",
    "EpGemmComm",
    "EpOracleComm",
    "EpPlan",
    "EpRoutes",
    "ExpertParallel",
    "ep_plan",
    "ep_routes",
    "shard_experts",
]

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


@dataclass
class EpRoutes:
    """Device-side routes of one MoE call on one rank, for the exchange fused into the GEMMs."""

    tokens: int
    top_k: int
    row_src: Tensor  # int32 [cap]: (source rank << 24) | source token of each received row, -1 = padding
    origin: Tensor  # int32 [cap]: (source rank << 24) | source slot of each received row, -1 = padding
    seg_start: Tensor  # int32 [EL + 1]: this rank's expert segments (multiples of 128)
    cap: int  # static bound on the received rows (multiple of 128)
    rows: int = 0  # rows actually received (seg_start[-1], at least 128), set by the forward


def ep_routes(indices: Tensor, num_experts: int, rank: int, world: int, group: Any = None) -> EpRoutes:
    """Routes for ``[T, k]`` global expert indices (one all-gather of the indices; device ops only).

    Every owner lays out expert ``e``'s rows as one 128-aligned segment holding the sources'
    rows in rank order and, within a source, in slot order: the layout of :func:`ep_plan`,
    computed here for every source so the owner knows where each of its rows comes from.
    """
    t, k = indices.shape
    s = t * k
    el = num_experts // world
    flat = indices.reshape(-1).to(torch.int32).contiguous()
    all_flat = _all_gather(flat, group, world) if world > 1 else flat.unsqueeze(0)  # [W, S]
    dev = flat.device
    g = all_flat.reshape(-1).long()  # global expert of every (source, slot)
    src = torch.arange(world, device=dev).repeat_interleave(s)
    slot = torch.arange(s, device=dev).repeat(world)
    key = src * num_experts + g
    counts = torch.bincount(key, minlength=world * num_experts)  # [(W, E)]
    tot = counts.view(world, num_experts).sum(0)
    padded = ((tot + 127) // 128 * 128).view(world, el)
    seg = padded.cumsum(1) - padded  # [owner, local expert] segment starts
    src_off = counts.view(world, num_experts).cumsum(0) - counts.view(world, num_experts)  # rows of lower sources
    key_start = counts.cumsum(0) - counts
    order = torch.argsort(key, stable=True)
    within = torch.empty_like(key)
    within[order] = torch.arange(world * s, device=dev) - key_start[key[order]]
    dest_row = seg.reshape(-1)[g] + src_off.reshape(-1)[key] + within
    cap = (world * s + 127) // 128 * 128 + 128 * el
    # rows bound for other owners land on a dump row past the end and are cut off
    at = torch.where(g // el == rank, dest_row, torch.full_like(dest_row, cap))
    code = (src << 24) | slot
    origin = torch.full((cap + 1,), -1, device=dev, dtype=torch.int64).scatter_(0, at, code)[:cap]
    row_src = torch.full((cap + 1,), -1, device=dev, dtype=torch.int64).scatter_(0, at, (src << 24) | (slot // k))[:cap]
    seg_start = torch.cat([seg[rank], (seg[rank, -1] + padded[rank, -1]).reshape(1)]).to(torch.int32)
    return EpRoutes(t, k, row_src.to(torch.int32), origin.to(torch.int32), seg_start, cap)


class EpGemmComm:
    """Owner of the native ``EpGemmGroup`` (send / recv rows and signals in IPC-mapped memory).

    Buffers grow on demand, collectively: every rank makes the same calls with the same sizes.
    """

    fused = True
    in_gemm = True

    def __init__(self, group: Any, timeout_s: float = 60.0) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = timeout_s
        self._g: Any = None
        self._cap = (0, 0, 0)

    def ensure(self, slots: int, cap: int, cols: int) -> Any:
        if self._g is not None and slots <= self._cap[0] and cap <= self._cap[1] and cols == self._cap[2]:
            return self._g
        from priml_b200.ops import native

        want = (max(slots, self._cap[0]), max(cap, self._cap[1]), cols)
        seen: list[Any] = [None] * self.world
        dist.all_gather_object(seen, want, group=self.group)
        if any(w != want for w in seen):
            raise ValueError(f"expert parallelism needs the same tokens per MoE call on every rank; got {seen}")
        if self._g is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        g = native().EpGemmGroup(self.rank, self.world, want[0], want[0], cols, want[1] // 128, self.timeout_s)
        handles: list[Any] = [None] * self.world
        dist.all_gather_object(handles, g.handles(), group=self.group)
        g.open(handles)
        self._g, self._cap = g, want
        return g


class _EpGemmMoE(torch.autograd.Function):
    """Routed expert SwiGLU with the token exchange inside the expert GEMMs (see ``ep_gemm.cu``)."""

    @staticmethod
    def forward(ctx, x: Tensor, weights: Tensor, up_w: Tensor, down_w: Tensor, routes: EpRoutes, comm: EpGemmComm):  # type: ignore[override]
        from priml_b200.ops.functional import bf16_shadow

        t, c = x.shape
        k = routes.top_k
        el, two_h, _ = up_w.shape
        h_dim = two_h // 2
        grp = comm.ensure(t * k, routes.cap, c)
        up16 = bf16_shadow(up_w).reshape(el * two_h, c)
        down16 = bf16_shadow(down_w).reshape(el * c, h_dim)
        grp.wait_send_free()
        grp.send_rows(t).copy_(x)
        # The received rows and the tensors kept for the backward are sized by this call's
        # real row count (one device read per layer) rather than by the static bound, which
        # is world times larger: at eight ranks the bound would not fit the saved activations.
        dev, cap = x.device, max(int(routes.seg_start[-1]), 128)
        routes.rows = cap
        x_priv = torch.empty(cap, c, device=dev, dtype=torch.bfloat16)
        h = torch.empty(cap, h_dim, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(cap, two_h, device=dev, dtype=torch.bfloat16)
        grp.pull_gemm(routes.row_src, routes.seg_start, up16, 3, two_h, h_dim, h, gu, x_priv)
        grp.push_gemm(h, routes.origin, routes.seg_start, down16, False, c)
        w32 = weights.float().contiguous()
        y = torch.empty(t, c, device=dev, dtype=torch.bfloat16)
        y_slots = torch.empty(t * k, c, device=dev, dtype=torch.bfloat16)
        grp.combine(t, k, w32, y, y_slots)
        ctx.save_for_backward(x_priv, h, gu, y_slots, w32, up16, down16)
        ctx.routes, ctx.comm, ctx.params, ctx.w_dtype = routes, comm, (up_w, down_w), weights.dtype
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        from priml_b200.ops import native
        from priml_b200.ops.grouped import _grad_into

        n = native()
        x_priv, h, gu, y_slots, w32, up16, down16 = ctx.saved_tensors
        routes, comm = ctx.routes, ctx.comm
        up_w, down_w = ctx.params
        t, k = w32.shape
        c = x_priv.shape[1]
        two_h = gu.shape[1]
        h_dim = two_h // 2
        dev, cap = dy.device, routes.rows
        grp = comm.ensure(t * k, routes.cap, c)
        dy16 = dy.to(torch.bfloat16).contiguous()
        grp.wait_send_free()
        dw = torch.empty(t, k, device=dev, dtype=torch.float32)
        n.ep_expand(dy16, w32, y_slots, grp.send_rows(t * k), dw)
        dy_priv = torch.empty(cap, c, device=dev, dtype=torch.bfloat16)
        dgu = torch.empty(cap, two_h, device=dev, dtype=torch.bfloat16)
        grp.pull_gemm(routes.origin, routes.seg_start, down16, 4, c, h_dim, dgu, gu, dy_priv)
        grp.push_gemm(dgu, routes.origin, routes.seg_start, up16, True, two_h)
        dx = torch.empty(t, c, device=dev, dtype=torch.bfloat16)
        grp.combine(t, k, None, dx, None)
        grads = []
        for param, a, b in ((up_w, dgu, x_priv), (down_w, dy_priv, h)):
            e_rows = param.shape[0] * param.shape[1]
            dst, acc, _ = _grad_into(param, e_rows)
            if dst is not None:
                n.grouped_gemm(a, b, dst, routes.seg_start, True, 2 if acc else 1, 1, 0)
                grads.append(None)
            else:
                out = torch.empty(e_rows, param.shape[2], device=dev, dtype=torch.float32)
                n.grouped_gemm(a, b, out, routes.seg_start, True, 1, 1, 0)
                grads.append(out.view_as(param).to(param.dtype))
        return dx, dw.to(ctx.w_dtype), grads[0], grads[1], None, None


class EpGemmDispatcher:
    """Installed on ``MoE.expert_parallel`` for ``comm="gemm"``: the exchange runs inside the expert GEMMs."""

    def __init__(self, comm: EpGemmComm) -> None:
        self.comm = comm

    def __call__(self, moe: nn.Module, xf: Tensor, weights: Tensor, indices: Tensor) -> Tensor:
        comm = self.comm
        routes = ep_routes(indices, moe.num_experts, comm.rank, comm.world, comm.group)
        experts = moe.experts
        y = _EpGemmMoE.apply(xf.to(torch.bfloat16).contiguous(), weights, experts.up_proj, experts.down_proj, routes, comm)
        return y.to(xf.dtype)


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
        mod.expert_parallel = EpGemmDispatcher(comm) if getattr(comm, "in_gemm", False) else EpDispatcher(comm)
        sharded += [ex.up_proj, ex.down_proj]
    return sharded


class ExpertParallel:
    """Strategy: experts sharded over the ``ep`` mesh axis (usually the data-parallel
    axis itself), every other parameter replicated with averaged gradients."""

    class Config(Fig["ExpertParallel"]):
        mesh_dim: str = "dp"
        timeout_s: float = 60.0
        comm: str = "auto"
        """``gemm`` (exchange inside the expert GEMMs; CUDA), ``fused`` (NVLink row-exchange kernels
        around separate grouped GEMMs; CUDA), ``oracle`` (all-gather), ``auto`` = gemm on CUDA."""

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
        if config.comm not in ("auto", "gemm", "fused", "oracle"):
            raise ValueError(f"comm must be auto, gemm, fused or oracle; got {config.comm!r}")
        if config.comm in ("gemm", "fused") and not use_cuda:
            raise RuntimeError("the fused expert exchange needs CUDA ranks")
        cls: Any = EpOracleComm
        if use_cuda and config.comm in ("auto", "gemm"):
            cls = EpGemmComm
        elif use_cuda and config.comm == "fused":
            cls = EpComm
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
