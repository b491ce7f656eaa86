"""Device-timed roofline benchmark of the fused tensor-parallel GEMMs vs NCCL + GEMM.

    torchrun --nproc-per-node N -m priml_b200.parallel.bench_tp [--tokens 8192]

Shapes: Llama-3-8B layers under sequence-parallel TP=N (tokens sharded across
ranks): column-parallel qkv / up projections (all-gather GEMM, K = 4096) and
row-parallel o / down projections (GEMM reduce-scatter, N = 4096). Each op is
timed with CUDA events (3 warm-up, 10 timed, max over ranks) against the
unfused baseline: NCCL all-gather then the tcgen05 GEMM, or the GEMM then NCCL
reduce-scatter. Roofline: max(FLOPs / measured bf16 peak, NVLink bytes / 770 GB/s).
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
    ap.add_argument("--tokens", type=int, default=8192)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))  # fmt: skip
    from priml_b200.cost import load_peaks
    from priml_b200.ops import native
    from priml_b200.ops.functional import gemm

    n = native()
    peak = load_peaks().bf16_tflops * 1e12
    M = args.tokens
    ms = M // world
    d, ffn, kv = 4096, 14336, 1024
    cases = {"qkv": ("ag", (d + 2 * kv) // world, d), "up": ("ag", 2 * ffn // world, d),
             "o": ("rs", d, d // world), "down": ("rs", d, ffn // world)}  # fmt: skip
    kmax = max(k for _, _, k in cases.values())
    nmax = max(nn for _, nn, _ in cases.values())
    grp = n.TpGroup(rank, world, ms * kmax, world * ms * nmax, (world - 1) * ms // 128, 30.0)
    handles: list = [None] * world
    dist.all_gather_object(handles, grp.handles())
    grp.open(handles)
    res = {}
    for name, (kind, N, K) in cases.items():
        w = (torch.randn(N, K, device="cuda") / K**0.5).to(torch.bfloat16)
        flops = 2.0 * M * N * K
        if kind == "ag":
            x = torch.randn(ms, K, device="cuda").to(torch.bfloat16)
            c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            a_full = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)

            def fused() -> None:
                grp.wait_shard_free()
                grp.shard()[: ms * K].view(ms, K).copy_(x)
                grp.ag_gemm(w, False, ms, K, c, a_full)

            def base() -> None:
                dist.all_gather_into_tensor(a_full, x)
                gemm(a_full, w, out=c)

            link = (world - 1) / world * M * K * 2
        else:
            a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
            out = torch.empty(ms, N, device="cuda", dtype=torch.bfloat16)
            part = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

            def fused() -> None:
                grp.gemm_rs(a, w, False, out)

            def base() -> None:
                gemm(a, w, out=part)
                dist.reduce_scatter_tensor(out, part)

            link = (world - 1) / world * M * N * 2
        tf, tb = _time(fused), _time(base)
        roof = max(flops / peak, link / NVLINK) * 1e3
        res[name] = {"kind": kind, "M": M, "N": N, "K": K, "fused_ms": round(tf, 4), "nccl_plus_gemm_ms": round(tb, 4),
                     "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / tf, 3)}  # fmt: skip
    status = int(n.read_status(True))
    if rank == 0:
        print(json.dumps({"world": world, "tokens": M, "cases": res, "status": status}), flush=True)
    del grp
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
