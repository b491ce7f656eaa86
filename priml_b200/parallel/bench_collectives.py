"""Device-timed roofline benchmark of the fused peer-memory collectives.

    torchrun --nproc-per-node N -m priml_b200.parallel.bench_collectives [--params 1.24e9]

For a model of ``--params`` parameters sharded over N ranks it times, with CUDA
events on the launching stream (warm-up first, max over ranks):

* ``rs_bucket`` over the whole fp32 gradient (one bucket per 64 Mi elements),
  vs NCCL ``reduce_scatter_tensor`` (fp32, average) of the same buffer;
* ``adamw_scatter`` (AdamW on the local shard + bf16 stores into every rank's
  weight copy), vs NCCL ``all_gather_into_tensor`` of the bf16 shard alone
  (the NCCL baseline still needs a separate optimizer kernel on top).

Roofline: the bytes that must cross NVLink per rank -- ``(N-1)/N * 4`` bytes per
parameter in for the reduce-scatter, ``(N-1)/N * 2`` out for the all-gather --
over the measured 770 GB/s per direction, and the local HBM bytes over the
measured copy bandwidth; the slower of the two is the target time.
Prints one JSON line from rank 0.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy, per direction per GPU


def _time(fn, iters: int, warmup: int = 3) -> float:  # noqa: ANN001
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
    ap.add_argument("--params", type=float, default=1.24e9)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--reduce-blocks", type=int, default=48)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))  # fmt: skip
    from priml_b200.cost import load_peaks
    from priml_b200.ops import native

    n = native()
    bucket = 64 * 1024 * 1024
    nb = max(1, int(args.params) // bucket)
    total = nb * bucket
    shard = bucket // world
    pg = n.PeerGroup(rank, world, total, total)
    handles: list = [None] * world
    dist.all_gather_object(handles, pg.handles())
    pg.open(handles)
    pg.grad().normal_()
    out = torch.empty(nb * shard, device="cuda")
    partial = torch.zeros(nb, args.reduce_blocks, device="cuda")
    epoch = [1]

    def rs() -> None:
        for b in range(nb):
            pg.reduce_scatter(b, b * bucket, shard, out[b * shard : (b + 1) * shard], partial[b], epoch[0],
                              1.0 / world, 30.0)  # fmt: skip
        epoch[0] += 1

    t_rs = _time(rs, args.iters)
    full = pg.grad()
    rs_out = torch.empty(total // world, device="cuda")
    t_nccl_rs = _time(lambda: dist.reduce_scatter_tensor(rs_out, full, op=dist.ReduceOp.AVG), args.iters)

    local = nb * shard
    master = torch.randn(local, device="cuda")
    m1 = torch.zeros(local, device="cuda")
    m2 = torch.zeros(local, device="cuda")
    segs = torch.tensor([[b * shard, b * bucket + rank * shard, 0] for b in range(nb)], dtype=torch.int64,
                        device="cuda")  # fmt: skip
    clip = torch.ones(1, device="cuda")
    hyper = [[1e-4], [0.9], [0.95], [1e-8], [0.1], [0.1], [0.05]]
    blocks = 2 * torch.cuda.get_device_properties(0).multi_processor_count
    target = [0]

    def adamw() -> None:
        pg.adamw_scatter(segs, master, m1, m2, out, clip, hyper, blocks)
        target[0] += world * blocks
        pg.barrier(target[0], 30.0)

    t_adam = _time(adamw, args.iters)
    shard16 = master.to(torch.bfloat16)
    gathered = torch.empty(local * world, dtype=torch.bfloat16, device="cuda")
    t_nccl_ag = _time(lambda: dist.all_gather_into_tensor(gathered, shard16), args.iters)
    status = int(n.read_status(True))

    peaks = load_peaks()
    hbm = peaks.hbm_gbs
    frac = (world - 1) / world
    rs_link = frac * total * 4 / (NVLINK_GBS * 1e9) * 1e3  # ms
    rs_hbm = (total * 4 / world * world + local * 4) / (hbm * 1e9) * 1e3  # every rank's slice read once + shard write
    ag_link = frac * local * world * 2 / (NVLINK_GBS * 1e9) * 1e3
    ag_hbm = (local * 4 * 7 + local * world * 2) / (hbm * 1e9) * 1e3  # g,p,m,v read; p,m,v write; bf16 in
    res = {
        "world": world,
        "params": total,
        "reduce_scatter": {
            "fused_ms": round(t_rs, 3),
            "nccl_ms": round(t_nccl_rs, 3),
            "roofline_ms": round(max(rs_link, rs_hbm), 3),
            "frac_of_roofline": round(max(rs_link, rs_hbm) / t_rs, 3),
            "nvlink_in_gbs": round(frac * total * 4 / (t_rs * 1e-3) / 1e9, 1),
        },
        "adamw_allgather": {
            "fused_ms": round(t_adam, 3),
            "nccl_allgather_only_ms": round(t_nccl_ag, 3),
            "roofline_ms": round(max(ag_link, ag_hbm), 3),
            "frac_of_roofline": round(max(ag_link, ag_hbm) / t_adam, 3),
            "nvlink_out_gbs": round(frac * local * world * 2 / (t_adam * 1e-3) / 1e9, 1),
        },
        "nvlink_gbs_per_direction": NVLINK_GBS,
        "hbm_gbs": hbm,
        "status": status,
    }
    if rank == 0:
        print(json.dumps(res), flush=True)
    del pg
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
