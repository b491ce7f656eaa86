"""Expert GEMMs fused with the expert-parallel exchange (``ep_gemm.cu``) on one GPU.

A one-rank group runs the whole fused path: the up projection pulls its
rows from the send buffer by peer-style loads, the down projection's epilogue
stores its rows into the receive buffer, and the combine kernel sums them.
Forward and every gradient are checked against an fp32 PyTorch oracle of the
routed SwiGLU experts, on two calls in a row (the second exercises the
epoch handshakes on buffers the first one used). The 2-GPU exchange is
covered by ``test_expert_parallel_gpu.py``.
"""

from __future__ import annotations

import socket

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def one_rank_group():
    import torch.distributed as dist

    if dist.is_initialized():
        yield dist.group.WORLD
        return
    # gloo carries the host-side handshakes (buffer sizes, IPC handles); the exchange itself
    # runs in the kernels, so no NCCL communicator (and no watchdog thread) is involved
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_port()}", rank=0, world_size=1)
    try:
        yield dist.group.WORLD
    finally:
        dist.destroy_process_group()


def _oracle(x, w, idx, up, down):  # noqa: ANN001, ANN202
    """sum_j w[t, j] * down_e @ (silu(gate_e x) * up_e x) in fp32, e = idx[t, j]."""
    t, k = idx.shape
    h_dim = up.shape[1] // 2
    out = torch.zeros(t, x.shape[1], device=x.device, dtype=torch.float32)
    for j in range(k):
        e = idx[:, j]
        gu = torch.einsum("tc,thc->th", x, up[e])
        h = F.silu(gu[:, :h_dim]) * gu[:, h_dim:]
        out = out + w[:, j : j + 1] * torch.einsum("th,tch->tc", h, down[e])
    return out


def _err(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


@pytest.mark.parametrize("T,C,H,E,k", [(333, 256, 256, 8, 2), (1024, 512, 384, 16, 6)])
def test_ep_gemm_matches_fp32_oracle(one_rank_group, T, C, H, E, k) -> None:  # noqa: ANN001
    from priml_b200.ops import native
    from priml_b200.parallel.expert import EpGemmComm, _EpGemmMoE, ep_routes

    torch.manual_seed(0)
    comm = EpGemmComm(one_rank_group, timeout_s=5.0)
    dev = torch.device("cuda", 0)
    up = torch.nn.Parameter(torch.randn(E, 2 * H, C, device=dev) * C**-0.5)
    down = torch.nn.Parameter(torch.randn(E, C, H, device=dev) * H**-0.5)
    for call in range(2):
        x = torch.randn(T, C, device=dev).to(torch.bfloat16).requires_grad_()
        logits = torch.randn(T, E, device=dev)
        wts, idx = torch.topk(logits.softmax(-1), k, dim=-1)
        wts = wts.detach().requires_grad_()
        g = torch.randn(T, C, device=dev)
        routes = ep_routes(idx, E, 0, 1, one_rank_group)
        up.grad = down.grad = None
        y = _EpGemmMoE.apply(x, wts, up, down, routes, comm)
        (y.float() * g).sum().backward()
        torch.cuda.synchronize()
        assert int(native().read_status(True)) == 0, f"kernel status on call {call}"

        xr = x.detach().float().requires_grad_()
        wr = wts.detach().clone().requires_grad_()
        upr = up.detach().to(torch.bfloat16).float().requires_grad_()
        downr = down.detach().to(torch.bfloat16).float().requires_grad_()
        yr = _oracle(xr, wr, idx, upr, downr)
        (yr * g).sum().backward()
        for name, got, ref in (("y", y, yr), ("dx", x.grad, xr.grad), ("dw", wts.grad, wr.grad),
                               ("dup", up.grad, upr.grad), ("ddown", down.grad, downr.grad)):  # fmt: skip
            assert torch.isfinite(got.float()).all(), (name, call)
            assert _err(got, ref) < 3e-2, (name, call, _err(got, ref))


def test_ep_routes_cover_every_slot_once(one_rank_group) -> None:  # noqa: ANN001
    from priml_b200.parallel.expert import ep_routes

    torch.manual_seed(1)
    idx = torch.randint(0, 8, (100, 3), device="cuda")
    r = ep_routes(idx, 8, 0, 1, one_rank_group)
    seg = r.seg_start.tolist()
    assert all(s % 128 == 0 for s in seg) and seg[-1] <= r.cap
    got = r.origin[r.origin >= 0]
    assert sorted(got.tolist()) == list(range(300))
    # each received row sits in the segment of its slot's expert, and its token is slot // k
    rows = torch.nonzero(r.origin >= 0).flatten()
    slots = r.origin[rows].long()
    e = idx.reshape(-1)[slots]
    assert bool(((rows >= r.seg_start.long()[e]) & (rows < r.seg_start.long()[e + 1])).all())
    assert torch.equal(r.row_src[rows].long(), slots // 3)
