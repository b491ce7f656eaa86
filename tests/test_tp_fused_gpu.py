"""Fused all-gather GEMM / GEMM reduce-scatter over NVLink peer memory (2+ GPUs)."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                         device_id=torch.device("cuda", rank))  # fmt: skip
    try:
        from priml_b200.ops import native

        n = native()
        m_shard, K, N = 256, 384, 640
        grp = n.TpGroup(rank, world, m_shard * K, world * m_shard * N, (world - 1) * m_shard // 128, 10.0)
        handles = [None] * world
        torch.distributed.all_gather_object(handles, grp.handles())
        grp.open(handles)
        errs = []
        for it in range(3):
            g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
            x = torch.randn(m_shard, K, device="cuda", generator=g).to(torch.bfloat16)
            w = (torch.randn(N, K, device="cuda", generator=g) / K**0.5).to(torch.bfloat16)
            # all-gather GEMM (B K-major and N-major)
            grp.wait_shard_free()
            grp.shard()[: m_shard * K].view(m_shard, K).copy_(x)
            full = [torch.empty_like(x) for _ in range(world)]
            torch.distributed.all_gather(full, x)
            xf = torch.cat(full)
            ref = xf.float() @ w.float().t()
            c = torch.empty(world * m_shard, N, device="cuda", dtype=torch.bfloat16)
            a_full = torch.empty(world * m_shard, K, device="cuda", dtype=torch.bfloat16)
            for b_mn in (False, True):
                grp.wait_shard_free()
                grp.shard()[: m_shard * K].view(m_shard, K).copy_(x)
                a_full.fill_(float("nan"))
                grp.ag_gemm(w.t().contiguous() if b_mn else w, b_mn, m_shard, K, c, a_full)
                errs.append(float((c.float() - ref).abs().max() / ref.abs().max()))
                errs.append(0.0 if torch.equal(a_full, xf) else 1.0)  # the gathered rows, own shard included
            # GEMM reduce-scatter (B K-major and N-major)
            a = torch.randn(world * m_shard, K, device="cuda", generator=g).to(torch.bfloat16)
            part = a.float() @ w.float().t()
            torch.distributed.all_reduce(part)
            want = part[rank * m_shard : (rank + 1) * m_shard]
            for b_mn in (False, True):
                out = torch.empty(m_shard, N, device="cuda", dtype=torch.bfloat16)
                grp.gemm_rs(a, w.t().contiguous() if b_mn else w, b_mn, out)
                errs.append(float((out.float() - want).abs().max() / want.abs().max()))
        torch.cuda.synchronize()
        status = int(n.read_status(True))
        q.put((rank, errs, status))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc), -1))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_fused_gemms_match_nccl_reference() -> None:
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, status in res:
        assert isinstance(errs, list), (rank, errs)
        assert status == 0, (rank, status)
        assert max(errs) < 2e-2, (rank, errs)


def _train_rank(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))  # fmt: skip
    try:
        from priml_b200.loss import TokenCrossEntropy
        from priml_b200.models.presets import tiny_lm
        from priml_b200.optimizers import FusedAdamW
        from priml_b200.parallel import runtime
        from priml_b200.parallel.tp_fused import FusedSequenceParallel
        from priml_b200.train import TrainStep

        runtime.initialize_global_device_mesh(device=torch.device("cuda"), mesh_topology={"tp": world}, timeout_s=120)
        g = torch.Generator().manual_seed(0)
        batches = [torch.randint(0, 512, (4 * world, 65), generator=g) for _ in range(3)]
        res = {}
        for comm in ("oracle", "fused"):
            torch.manual_seed(0)
            step = TrainStep.Config(
                model=tiny_lm(),
                optimizer=FusedAdamW.Config(lr=3e-3, betas=(0.9, 0.95), weight_decay=0.1),
                loss=TokenCrossEntropy.Config(),
                parallelism=FusedSequenceParallel.Config(comm=comm),
                gradient_clip_norm=1.0,
                dtype_autocast=torch.bfloat16,
            ).make()
            losses = []
            for seq in batches:
                local = seq.chunk(world)[rank].cuda()
                out = step.train_step(tokens=local[:, :-1], targets=local[:, 1:])
                t = out["loss"].detach().float().mean()
                torch.distributed.all_reduce(t)
                losses.append(float(t) / world)
            res[comm] = (losses, float(step.last_grad_norm))
        from priml_b200.ops import native

        torch.cuda.synchronize()
        q.put((rank, res, int(native().read_status(True))))
    except Exception as exc:  # noqa: BLE001
        import traceback

        q.put((rank, repr(exc) + traceback.format_exc(), -1))
    finally:
        from priml_b200.parallel import runtime

        runtime.destroy_global_device_mesh()
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_training_fused_matches_oracle() -> None:
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_train_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, out, status in res:
        assert isinstance(out, dict), (rank, out)
        assert status == 0, (rank, status)
        (lo, no), (lf, nf) = out["oracle"], out["fused"]
        for a, b in zip(lf, lo, strict=True):
            assert abs(a - b) < 2e-2 * max(1.0, abs(b)), (lf, lo)
        assert abs(nf - no) < 5e-2 * max(1.0, no), (nf, no)
