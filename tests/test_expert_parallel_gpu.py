"""Expert parallelism vs the all-gather oracle (2 GPUs): the NVLink row-exchange kernels around
separate grouped GEMMs (``fused``) and the exchange inside the expert GEMMs (``gemm``)."""

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
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))  # fmt: skip
    try:
        from priml_b200.loss import TokenCrossEntropy
        from priml_b200.models.presets import tiny_moe_lm
        from priml_b200.ops import native
        from priml_b200.optimizers import FusedAdamW
        from priml_b200.parallel import runtime
        from priml_b200.parallel.expert import ExpertParallel
        from priml_b200.train import TrainStep

        runtime.initialize_global_device_mesh(device=torch.device("cuda"), mesh_topology={"dp": world}, timeout_s=120)
        g = torch.Generator().manual_seed(0)
        batches = [torch.randint(0, 512, (4 * world, 129), generator=g) for _ in range(3)]
        res = {}
        for comm in ("oracle", "fused", "gemm"):
            torch.manual_seed(0)
            step = TrainStep.Config(
                model=tiny_moe_lm(),
                optimizer=FusedAdamW.Config(lr=3e-3, betas=(0.9, 0.95), weight_decay=0.1),
                loss=TokenCrossEntropy.Config(),
                parallelism=ExpertParallel.Config(comm=comm),
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
def test_expert_parallel_fused_exchange_matches_oracle() -> None:
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, out, status in res:
        assert isinstance(out, dict), (rank, out)
        assert status == 0, (rank, status)
        lo, no = out["oracle"]
        for comm in ("fused", "gemm"):
            lf, nf = out[comm]
            for a, b in zip(lf, lo, strict=True):
                assert abs(a - b) < 2e-2 * max(1.0, abs(b)), (comm, lf, lo)
            assert abs(nf - no) < 5e-2 * max(1.0, no), (comm, nf, no)
