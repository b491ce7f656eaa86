"""Device-timed roofline benchmark of the expert GEMMs with the exchange inside them.

    torchrun --nproc-per-node N -m priml_b200.parallel.bench_ep [--tokens 8192]

Shape: one MoE layer of the MLA + MoE decoder (d_model 2048, 64 routed experts
of hidden 1408, top-6, uniform random routing) with the experts split over the
N ranks. Timed with CUDA events (3 warm-up, 10 timed, max over ranks):

* ``pull_up``   the up projection pulling its rows from the sources
  (``EpGemmGroup.pull_gemm``, SwiGLU epilogue), against the same grouped GEMM
  on rows already in place (``grouped_gemm``, epilogue 3);
* ``push_down`` the down projection storing its rows into the sources
  (``push_gemm``), against the grouped GEMM writing locally (epilogue 0);
* ``layer``     the whole fused forward (send-buffer fill, pull, push,
  weighted combine), against the peer-store exchange kernels around the two
  grouped GEMMs (``EpComm``).

Roofline: max(FLOPs / measured bf16 peak, NVLink bytes / 770 GB/s), where the
NVLink bytes are the rows that cross to or from other ranks ((N-1)/N of them
under uniform routing).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK = 770e9


def _time(fn, iters: int = 10, warmup: int = 3) -> float:  # noqa: ANN001
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192, help="tokens per rank")
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--top-k", type=int, default=6)
    ap.add_argument("--d-model", type=int, default=2048)
    ap.add_argument("--hidden", type=int, default=1408)
    args = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))  # fmt: skip
    from priml_b200.cost import load_peaks
    from priml_b200.ops import grouped_swiglu_mlp, native
    from priml_b200.parallel.expert import EpComm, EpGemmComm, _EpGemmMoE, ep_plan, ep_routes

    n = native()
    peak = load_peaks().bf16_tflops * 1e12
    T, E, k, C, H = args.tokens, args.experts, args.top_k, args.d_model, args.hidden
    el = E // world
    torch.manual_seed(rank)
    x = torch.randn(T, C, device="cuda").to(torch.bfloat16)
    wts, idx = torch.topk(torch.randn(T, E, device="cuda").softmax(-1), k, dim=-1)
    up = torch.randn(el, 2 * H, C, device="cuda") * C**-0.5
    down = torch.randn(el, C, H, device="cuda") * H**-0.5
    up16 = up.to(torch.bfloat16).reshape(el * 2 * H, C)
    down16 = down.to(torch.bfloat16).reshape(el * C, H)

    comm = EpGemmComm(dist.group.WORLD, timeout_s=30.0)
    routes = ep_routes(idx, E, rank, world, dist.group.WORLD)
    cap = max(int(routes.seg_start[-1]), 128)  # rows actually received
    grp = comm.ensure(T * k, routes.cap, C)
    x_priv = torch.empty(cap, C, device="cuda", dtype=torch.bfloat16)
    h = torch.empty(cap, H, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(cap, 2 * H, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(T, C, device="cuda", dtype=torch.bfloat16)
    y_local = torch.empty(cap, C, device="cuda", dtype=torch.bfloat16)
    grp.send_rows(T).copy_(x)
    rows = int(routes.seg_start[-1])  # rows this rank's experts receive (real + segment padding)
    received = int((routes.origin >= 0).sum())
    remote = int(((routes.origin >= 0) & ((routes.origin >> 24) != rank)).sum())

    def pull() -> None:
        grp.wait_send_free()
        grp.pull_gemm(routes.row_src, routes.seg_start, up16, 3, 2 * H, H, h, gu, x_priv)

    def up_local() -> None:
        n.grouped_gemm(x_priv, up16, h, routes.seg_start, False, 3, 0, 2 * H, gu, H)

    def push() -> None:
        grp.push_gemm(h, routes.origin, routes.seg_start, down16, False, C)
        grp.combine(T, k, wts, y, None)  # frees the recv buffer for the next push

    def down_local() -> None:
        n.grouped_gemm(h, down16, y_local, routes.seg_start, False, 0, 0, C)

    w32 = wts.float().contiguous()
    upp = torch.nn.Parameter(up)
    downp = torch.nn.Parameter(down)

    def layer() -> None:
        with torch.no_grad():
            _EpGemmMoE.apply(x, w32, upp, downp, routes, comm)

    old = EpComm(dist.group.WORLD, timeout_s=30.0)

    def layer_exchange_kernels() -> None:
        from priml_b200.parallel.expert import _ToExperts, _ToSources

        with torch.no_grad():
            plan = ep_plan(idx, E, rank, world, dist.group.WORLD)
            xp = _ToExperts.apply(x, plan, old)
            yp = grouped_swiglu_mlp(xp, upp, downp, plan.seg_start)
            ys = _ToSources.apply(yp.to(torch.bfloat16), plan, old)
            (ys.float() * w32.reshape(-1, 1)).view(T, k, -1).sum(1)

    f_up = 2.0 * rows * 2 * H * C
    f_down = 2.0 * rows * C * H
    link_in = remote * C * 2
    res = {}
    for name, fused, base, flops, link in (
        ("pull_up", pull, up_local, f_up, link_in),
        ("push_down", push, down_local, f_down, link_in),
        ("layer", layer, layer_exchange_kernels, f_up + f_down, 2 * link_in),
    ):
        tf, tb = _time(fused), _time(base)
        roof = max(flops / peak, link / NVLINK) * 1e3
        res[name] = {"fused_ms": round(tf, 4), "baseline_ms": round(tb, 4), "roofline_ms": round(roof, 4),
                     "frac_of_roofline": round(roof / tf, 3), "tflops": round(flops / tf / 1e9, 1)}  # fmt: skip
    status = int(n.read_status(True))
    if rank == 0:
        print(json.dumps({"world": world, "tokens_per_rank": T, "experts": E, "top_k": k, "d_model": C, "hidden": H,
                          "rows_received": received, "rows_remote": remote, "segment_rows": rows, "cases": res,
                          "baselines": {"pull_up": "grouped GEMM on rows in place", "push_down": "grouped GEMM, local store",
                                        "layer": "peer-store exchange kernels around the grouped GEMMs"},
                          "status": status}), flush=True)  # fmt: skip
    del grp, comm, old
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
