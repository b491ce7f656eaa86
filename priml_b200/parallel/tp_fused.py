"""Sequence-parallel tensor parallelism on the fused NVLink GEMMs.

Same sharding as Megatron-style TP with sequence parallelism (the reference's
DTensor plan: ``priml/train/tensor_parallel.py:101-224``, column/row styles
declared by ``priml/model/linear.py:154-199`` and ``priml/model/swiglu.py:255-278``),
with the activation shards laid out for the fused kernels:

* Between TP regions every rank holds a contiguous block of rows of the
  flattened ``[batch * seq, channels]`` activations: its own micro-batch. From
  the data side the strategy therefore looks exactly like data parallelism
  (every rank loads different sequences), and norms, residual adds, the
  embedding and the loss run on local rows.
* Column-parallel layers (``shard="colwise"``: attention qkv, SwiGLU up/gate)
  gather the rows of all TP ranks inside ONE kernel with the GEMM
  (``tp_ag_gemm``: peer rows are pulled over NVLink tile by tile while the
  tensor cores work on the rows already present) and keep the gathered input
  for the weight gradient. Their input gradient is a fused GEMM
  reduce-scatter.
* Row-parallel layers (``shard="rowwise"``: attention output, SwiGLU down)
  run the GEMM with the reduce-scatter fused into its epilogue
  (``tp_gemm_rs``); their backward is a fused all-gather GEMM whose gathered
  output gradient also feeds the weight gradient.

Gradients: a sharded weight sees the tokens of every TP rank, a replicated
parameter (norms, embeddings, head) only its own rank's. With each rank's loss
the mean over its rows, the global objective is the mean over ranks, so
replicated gradients are averaged over all ranks (one flattened all-reduce
per optimizer step) and sharded gradients are summed over the
data-parallel axis and divided by the world size. The
gradient-norm clip sums the squares of the sharded gradients across the TP
ranks and counts the replicated ones once.

Without CUDA (gloo ranks) the same layers run an oracle communicator built on
``torch.distributed`` (all-gather + matmul, matmul + all-reduce slice).
"""

from __future__ import annotations

import logging
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor, nn

from priml_b200.config import Fig
from priml_b200.parallel.runtime import global_device_mesh
from priml_b200.parallel.strategies import place

__all__ = [
    "FusedSequenceParallel",
    "SPColumnLinear",
    "SPRowLinear",
    "TpComm",
    "TpGradSync",
    "TpOracleComm",
]

log = logging.getLogger(__name__)


# --------------------------------------------------------------------------- communicators
class TpComm:
    """Fused NVLink all-gather GEMM / GEMM reduce-scatter over one TP process group.

    Owns one native ``TpGroup`` (IPC shard, receive slots and signal words on
    every rank). Buffers grow on demand; every rank issues the same calls with
    the same shapes in the same order, so a growth is itself collective.
    """

    fused = True

    def __init__(self, group: dist.ProcessGroup | None, timeout_s: float = 60.0) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = timeout_s
        self._g: Any = None
        self._cap = (0, 0, 0)

    def _ensure(self, shard_elems: int, slot_elems: int, chunks: int) -> Any:
        cap = self._cap
        if self._g is not None and shard_elems <= cap[0] and slot_elems <= cap[1] and chunks <= cap[2]:
            return self._g
        from priml_b200.ops import native

        want = (max(shard_elems, cap[0]), max(slot_elems, cap[1]), max(chunks, cap[2], 1))
        if self._g is not None:
            # peers may still read the old buffers until every rank is here
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        g = native().TpGroup(self.rank, self.world, want[0], want[1], want[2], self.timeout_s)
        handles: list[Any] = [None] * self.world
        dist.all_gather_object(handles, g.handles(), group=self.group)
        g.open(handles)
        self._g, self._cap = g, want
        return g

    def ag_gemm(self, x2: Tensor, w16: Tensor, b_mn: bool) -> tuple[Tensor, Tensor]:
        """``(AllGather_rows(x2) @ B^T, gathered x2)``; B = ``w16`` ``[N, K]`` (``[K, N]`` if ``b_mn``)."""
        m_s, k = x2.shape
        n = w16.shape[1] if b_mn else w16.shape[0]
        g = self._ensure(m_s * k, 0, (self.world - 1) * (m_s // 128))
        g.wait_shard_free()
        g.shard()[: m_s * k].view(m_s, k).copy_(x2)
        y = torch.empty(self.world * m_s, n, device=x2.device, dtype=torch.bfloat16)
        x_full = torch.empty(self.world * m_s, k, device=x2.device, dtype=torch.bfloat16)
        g.ag_gemm(w16, b_mn, m_s, k, y, x_full)
        return y, x_full

    def gemm_rs(self, a2: Tensor, w16: Tensor, b_mn: bool) -> Tensor:
        """Rows of this rank of ``sum_ranks(a2 @ B^T)``."""
        m, _ = a2.shape
        n = w16.shape[1] if b_mn else w16.shape[0]
        g = self._ensure(0, m * n, 0)
        out = torch.empty(m // self.world, n, device=a2.device, dtype=torch.bfloat16)
        g.gemm_rs(a2, w16, b_mn, out)
        return out

    @staticmethod
    def supports(rows: int, k: int, n: int) -> bool:
        return rows % 128 == 0 and k % 8 == 0 and n % 8 == 0


class TpOracleComm:
    """``torch.distributed`` reference of :class:`TpComm` (any backend, any device)."""

    fused = False

    def __init__(self, group: dist.ProcessGroup | None, timeout_s: float = 60.0) -> None:
        del timeout_s
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def _gather(self, x: Tensor) -> Tensor:
        parts = [torch.empty_like(x) for _ in range(self.world)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts)

    def ag_gemm(self, x2: Tensor, w: Tensor, b_mn: bool) -> tuple[Tensor, Tensor]:
        x_full = self._gather(x2)
        w = w.to(x_full.dtype)
        return (x_full @ w if b_mn else x_full @ w.t()), x_full

    def gemm_rs(self, a2: Tensor, w: Tensor, b_mn: bool) -> Tensor:
        w = w.to(a2.dtype)
        part = (a2 @ w if b_mn else a2 @ w.t()).contiguous()
        dist.all_reduce(part, group=self.group)
        m_s = a2.shape[0] // self.world
        return part[self.rank * m_s : (self.rank + 1) * m_s].contiguous()

    @staticmethod
    def supports(rows: int, k: int, n: int) -> bool:
        del rows, k, n
        return True


# --------------------------------------------------------------------------- autograd
def _operand(x: Tensor, comm: Any) -> Tensor:
    if comm.fused:
        from priml_b200.ops.functional import _as_bf16_2d

        return _as_bf16_2d(x)
    return x.reshape(-1, x.shape[-1])


def _weight(w: Tensor, comm: Any, dtype: torch.dtype) -> Tensor:
    if comm.fused:
        from priml_b200.ops.functional import bf16_shadow

        return bf16_shadow(w)
    return w.to(dtype)


def _wgrad(weight: Tensor, w_op: Tensor, dy2: Tensor, x2: Tensor, comm: Any) -> Tensor | None:
    if comm.fused:
        from priml_b200.ops.functional import grad_sink, wgrad

        return wgrad(weight if grad_sink(weight) is not None else w_op, dy2, x2, weight.dtype)
    return (dy2.t().float() @ x2.float()).to(weight.dtype)


class _ColumnSP(torch.autograd.Function):
    """``y[M, N_l] = AllGather(x[m_s, K]) @ W_l^T``; backward: ``dx = RS(dy @ W_l)``, ``dW_l = dy^T x_full``."""

    @staticmethod
    def forward(ctx, x2: Tensor, weight: Tensor, comm: Any) -> Tensor:  # type: ignore[override]
        w = _weight(weight, comm, x2.dtype)
        y, x_full = comm.ag_gemm(x2, w, False)
        ctx.save_for_backward(x_full, w)
        ctx.comm, ctx.weight, ctx.x_dtype = comm, weight, x2.dtype
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x_full, w = ctx.saved_tensors
        comm = ctx.comm
        dy2 = _operand(dy, comm)
        dx = comm.gemm_rs(dy2, w, True).to(ctx.x_dtype) if ctx.needs_input_grad[0] else None
        dw = _wgrad(ctx.weight, w, dy2, x_full, comm) if ctx.needs_input_grad[1] else None
        return dx, dw, None


class _RowSP(torch.autograd.Function):
    """``y[m_s, N] = ReduceScatter(x[M, K_l] @ W_l^T)``; backward: ``dx = AllGather(dy) @ W_l``, ``dW_l = dy_full^T x``."""

    @staticmethod
    def forward(ctx, x2: Tensor, weight: Tensor, comm: Any) -> Tensor:  # type: ignore[override]
        w = _weight(weight, comm, x2.dtype)
        y = comm.gemm_rs(x2, w, False)
        ctx.save_for_backward(x2, w)
        ctx.comm, ctx.weight, ctx.x_dtype = comm, weight, x2.dtype
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, w = ctx.saved_tensors
        comm = ctx.comm
        dy2 = _operand(dy, comm)
        dx, dy_full = comm.ag_gemm(dy2, w, True)
        dx = dx.to(ctx.x_dtype) if ctx.needs_input_grad[0] else None
        dw = _wgrad(ctx.weight, w, dy_full, x2, comm) if ctx.needs_input_grad[1] else None
        return dx, dw, None


# --------------------------------------------------------------------------- layers
class SPColumnLinear(nn.Module):
    """Column-parallel projection on local rows: ``[b, ..., K] -> [tp*b, ..., *out_shape]``.

    ``weight`` is this rank's slice (``[N_l, K]``, or ``[E_l, c, K]`` for an
    ensemble/per-head projection); the output covers the rows of every TP rank
    in rank order.
    """

    def __init__(self, weight: Tensor, comm: Any) -> None:
        super().__init__()
        self.weight = nn.Parameter(weight.detach().clone())
        self.bias = None
        self.comm = comm
        self.shard = None  # already placed: not a target for another plan

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        w = self.weight
        w2 = w.reshape(-1, w.shape[-1])
        x2 = _operand(x, self.comm)
        y = _ColumnSP.apply(x2, w2, self.comm)
        lead = (x.shape[0] * self.comm.world, *x.shape[1:-1])
        return y.view(*lead, *w.shape[:-1])


class SPRowLinear(nn.Module):
    """Row-parallel projection back to local rows: ``[tp*b, ..., K_l] -> [b, ..., N]``."""

    def __init__(self, weight: Tensor, comm: Any) -> None:
        super().__init__()
        self.weight = nn.Parameter(weight.detach().clone())
        self.bias = None
        self.comm = comm
        self.shard = None

    def forward(self, x: Tensor, *args: Any, **kwargs: Any) -> Tensor:
        del args, kwargs
        x2 = _operand(x, self.comm)
        y = _RowSP.apply(x2, self.weight, self.comm)
        lead = (x.shape[0] // self.comm.world, *x.shape[1:-1])
        return y.view(*lead, self.weight.shape[0])


def _slice_rows(w: Tensor, rank: int, tp: int, dim: int = 0) -> Tensor:
    n = w.shape[dim]
    if n % tp:
        raise ValueError(f"dimension {n} is not divisible by the tensor-parallel size {tp}")
    return w.narrow(dim, rank * (n // tp), n // tp)


def _shard_attention(mod: nn.Module, comm: Any) -> None:
    from priml_b200.models.linear import EnsembleLinear

    tp, r = comm.world, comm.rank
    if getattr(mod, "split_qkv_projection", False) or getattr(mod, "norm_out", None) is not None:
        raise NotImplementedError("fused sequence parallelism needs a fused qkv projection and no full-width out norm")
    if not isinstance(mod.proj_qkv, EnsembleLinear) or mod.proj_qkv.bias is not None or mod.proj_out.bias is not None:
        raise NotImplementedError("fused sequence parallelism supports bias-free attention projections")
    h, kv = mod.heads, mod.num_heads_kv
    if h % tp or kv % tp:
        raise ValueError(f"heads={h} / kv heads={kv} must be divisible by the tensor-parallel size {tp}")
    w = mod.proj_qkv.weight.data  # [h + 2 kv, c, D]: q heads, k heads, v heads
    parts = (w[:h], w[h : h + kv], w[h + kv :])
    local = torch.cat([_slice_rows(p, r, tp) for p in parts])
    mod.proj_qkv = SPColumnLinear(local, comm)
    mod.proj_out = SPRowLinear(_slice_rows(mod.proj_out.weight.data, r, tp, dim=1), comm)
    mod.heads, mod.num_heads_kv = h // tp, kv // tp


def _shard_swiglu(mod: nn.Module, comm: Any) -> None:
    tp, r = comm.world, comm.rank
    if getattr(mod, "split_gate_projection", False) or getattr(mod, "norm", None) is not None:
        raise NotImplementedError("fused sequence parallelism needs a fused gate/up projection without a gate norm")
    if mod.up_proj.bias is not None or mod.down_proj.bias is not None:
        raise NotImplementedError("fused sequence parallelism supports bias-free SwiGLU projections")
    w = mod.up_proj.weight.data
    if getattr(mod, "gate", True):
        gate, up = w.chunk(2, dim=0)
        local = torch.cat([_slice_rows(gate, r, tp), _slice_rows(up, r, tp)])
    else:
        local = _slice_rows(w, r, tp)
    mod.up_proj = SPColumnLinear(local, comm)
    mod.down_proj = SPRowLinear(_slice_rows(mod.down_proj.weight.data, r, tp, dim=1), comm)


def shard_sequence_parallel(model: nn.Module, comm: Any) -> list[nn.Parameter]:
    """Swap the projections of every attention and SwiGLU block for fused
    sequence-parallel layers; returns the sharded parameters.

    Every other module stays replicated and runs on this rank's rows (whole
    sequences), i.e. data-parallel inside the TP group, which is exact for any
    row- or sequence-local block (norms, embeddings, MoE, recurrent mixers)."""
    from priml_b200.models.attention import SelfAttention
    from priml_b200.models.swiglu import SwiGLU

    done: set[int] = set()
    for _, mod in list(model.named_modules()):
        if id(mod) in done:
            continue
        if isinstance(mod, SelfAttention):
            _shard_attention(mod, comm)
        elif isinstance(mod, SwiGLU):
            _shard_swiglu(mod, comm)
        else:
            continue
        done.update(id(m) for m in mod.modules())
    sharded = []
    for mod in model.modules():
        if isinstance(mod, (SPColumnLinear, SPRowLinear)):
            sharded.append(mod.weight)
    return sharded


# --------------------------------------------------------------------------- gradients
class TpGradSync:
    """Gradient reductions of the sequence-parallel layout (see the module docstring).

    Backward only marks the gradients dirty; :meth:`wait` (called before the
    clip norm and the optimizer step, i.e. once per accumulation window) sums
    the replicated gradients over every rank and the sharded ones over the
    data-parallel axis, each group flattened into one collective, and applies
    the 1/world scale. No collective runs while the fused GEMMs, whose CTAs
    wait on their peers, are in flight.
    """

    def __init__(self, model: nn.Module, sharded: list[nn.Parameter], dp_group: Any, world: int) -> None:
        self.sharded_ids = {id(p) for p in sharded}
        self.dp_group = dp_group  # None: no data-parallel axis
        self.world = world
        self.scale = 1.0 / world
        self.dirty = False
        self.params = [p for p in model.parameters() if p.requires_grad]
        for p in self.params:
            p.register_post_accumulate_grad_hook(self._hook)

    def _hook(self, p: Tensor) -> None:
        del p
        self.dirty = True

    @staticmethod
    def _reduce(grads: list[Tensor], group: Any) -> None:
        if not grads:
            return
        from torch._utils import _flatten_dense_tensors, _unflatten_dense_tensors

        for dtype in sorted({g.dtype for g in grads}, key=str):
            same = [g for g in grads if g.dtype == dtype]
            flat = _flatten_dense_tensors(same)
            dist.all_reduce(flat, group=group)
            for g, r in zip(same, _unflatten_dense_tensors(flat, same), strict=True):
                g.copy_(r)

    def wait(self) -> None:
        if not self.dirty:
            return
        self.dirty = False
        repl = [p.grad for p in self.params if p.grad is not None and id(p) not in self.sharded_ids]
        shard = [p.grad for p in self.params if p.grad is not None and id(p) in self.sharded_ids]
        if self.world > 1:
            self._reduce(repl, None)
        if self.dp_group is not None and dist.get_world_size(self.dp_group) > 1:
            self._reduce(shard, self.dp_group)
        if repl or shard:
            torch._foreach_mul_(repl + shard, self.scale)  # noqa: SLF001


class TpOptimizer:
    """Optimizer proxy: completes the gradient reductions before the norm and the step,
    and computes the clip norm over the TP-sharded layout."""

    def __init__(self, base: Any, sync: TpGradSync, tp_group: Any) -> None:
        object.__setattr__(self, "base", base)
        object.__setattr__(self, "sync", sync)
        object.__setattr__(self, "tp_group", tp_group)

    def __getattr__(self, name: str) -> Any:
        return getattr(self.base, name)

    def __setattr__(self, name: str, value: Any) -> None:
        setattr(self.base, name, value)

    def fused_grad_norm(self, max_norm: float) -> tuple[Tensor, Tensor]:
        self.sync.wait()
        sharded, repl = [], []
        for p in self.sync.params:
            if p.grad is not None:
                (sharded if id(p) in self.sync.sharded_ids else repl).append(p.grad)
        dev = (sharded or repl)[0].device

        def sq(gs: list[Tensor]) -> Tensor:
            if not gs:
                return torch.zeros((), device=dev)
            return torch.stack([n.float() ** 2 for n in torch._foreach_norm(gs)]).sum()  # noqa: SLF001

        s = sq(sharded)
        if self.tp_group is not None and dist.get_world_size(self.tp_group) > 1:
            dist.all_reduce(s, group=self.tp_group)
        norm = (s + sq(repl)).sqrt()
        clip = (max_norm / (norm + 1e-6)).clamp(max=1.0)
        if not hasattr(self.base, "fused_grad_norm"):
            torch._foreach_mul_(sharded + repl, clip)  # noqa: SLF001
        return norm, clip

    def step(self, closure: Any = None) -> Any:
        self.sync.wait()
        return self.base.step(closure) if closure is not None else self.base.step()

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.base.zero_grad(set_to_none=set_to_none)

    def state_dict(self) -> dict[str, Any]:
        return self.base.state_dict()

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        self.base.load_state_dict(sd)


# --------------------------------------------------------------------------- strategy
class FusedSequenceParallel:
    """Strategy: tensor parallelism over ``tp`` with the fused NVLink GEMMs
    (plus plain data parallelism over ``dp`` when the mesh has it)."""

    class Config(Fig["FusedSequenceParallel"]):
        mesh_dim: str = "tp"
        dp_mesh_dim: str = "dp"
        timeout_s: float = 60.0
        comm: str = "auto"
        """``fused`` (NVLink kernels; CUDA), ``oracle`` (torch.distributed), ``auto`` = fused on CUDA."""

    def __init__(self, config: Config | None = None) -> None:
        config = config or FusedSequenceParallel.Config()
        mesh = global_device_mesh()
        if mesh is None:
            raise RuntimeError("FusedSequenceParallel requires the MultiProcess runtime.")
        names = mesh.mesh_dim_names or ()
        if config.mesh_dim not in names:
            raise ValueError(f"Mesh dimension {config.mesh_dim!r} not in {names}.")
        self.mesh = mesh
        self.tp_group = mesh[config.mesh_dim].get_group()
        self.dp_group = mesh[config.dp_mesh_dim].get_group() if config.dp_mesh_dim in names else None
        use_cuda = mesh.device_type == "cuda"
        self.device = torch.device("cuda", torch.cuda.current_device()) if use_cuda else torch.device(mesh.device_type)
        if config.comm not in ("auto", "fused", "oracle"):
            raise ValueError(f"comm must be auto, fused or oracle; got {config.comm!r}")
        if config.comm == "fused" and not use_cuda:
            raise RuntimeError("the fused tensor-parallel GEMMs need CUDA ranks")
        comm_cls = TpComm if (use_cuda and config.comm != "oracle") else TpOracleComm
        self.comm = comm_cls(self.tp_group, config.timeout_s)
        self.sync: TpGradSync | None = None

    def __call__(self, model: nn.Module) -> nn.Module:
        model = place(model, self.device)
        sharded = shard_sequence_parallel(model, self.comm)
        model.to(self.device)
        self.sync = TpGradSync(model, sharded, self.dp_group, dist.get_world_size())
        log.info("Fused sequence parallelism: tp=%d, %d sharded weights.", self.comm.world, len(sharded))
        return model

    def build_optimizer(self, make: Any, model: nn.Module) -> Any:
        assert self.sync is not None, "apply the strategy to the model first"
        base = make([p for p in model.parameters() if p.requires_grad])
        return TpOptimizer(base, self.sync, self.tp_group)

