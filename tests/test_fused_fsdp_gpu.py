"""Fused reduce-scatter / AdamW / all-gather kernels over peer memory (CUDA)."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _native():  # noqa: ANN202
    from priml_b200.ops import native

    return native()


def test_reduce_scatter_and_adamw_scatter_single_rank_match_torch() -> None:
    from priml_b200.ops import reference

    torch.manual_seed(0)
    n = 4096 * 3
    pg = _native().PeerGroup(0, 1, n, n)
    pg.open([pg.handles()])
    grad = pg.grad()
    grad.copy_(torch.randn(n, device="cuda"))
    # bucket 1 = elements [4096, 8192)
    out = torch.empty(4096, device="cuda")
    partial = torch.zeros(8, device="cuda")
    pg.reduce_scatter(1, 4096, 4096, out, partial, 1, 0.5, 5.0)
    torch.cuda.synchronize()
    assert torch.equal(out, grad[4096:8192] * 0.5)
    assert torch.allclose(partial.sum(), (out.double() ** 2).sum().float(), rtol=1e-5)

    master = torch.randn(4096, device="cuda")
    m1 = torch.randn(4096, device="cuda") * 0.1
    m2 = torch.rand(4096, device="cuda") * 0.01
    ref_p, ref_m, ref_v = master.clone(), m1.clone(), m2.clone()
    norm = torch.zeros(1, device="cuda")
    clip = torch.zeros(1, device="cuda")
    pg.norm_exchange(partial, 1, 1.0, norm, clip, 5.0)
    segs = torch.tensor([[0, 4096, 0], [2048, 6144, 1]], dtype=torch.int64, device="cuda")
    hyper = [[1e-3, 2e-3], [0.9, 0.9], [0.95, 0.95], [1e-8, 1e-8], [0.1, 0.0], [0.1, 0.1], [0.05, 0.05]]
    pg.adamw_scatter(segs, master, m1, m2, out, clip, hyper, 16)
    pg.barrier(16, 5.0)
    torch.cuda.synchronize()
    assert int(_native().read_status(True)) == 0
    true_norm = float((out.double() ** 2).sum().sqrt())
    assert abs(float(norm) - true_norm) < 1e-4 * true_norm
    c = min(1.0, 1.0 / (true_norm + 1e-6))
    g = out * float(clip)
    for lo, hi, lr, wd in ((0, 2048, 1e-3, 0.1), (2048, 4096, 2e-3, 0.0)):
        p_, m_, v_ = ref_p[lo:hi].clone(), ref_m[lo:hi].clone(), ref_v[lo:hi].clone()
        reference.adamw_([p_], [g[lo:hi]], [m_], [v_], step=1, lr=lr, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=wd)
        assert torch.allclose(master[lo:hi], p_, rtol=1e-6, atol=1e-7)
        assert torch.allclose(m1[lo:hi], m_, rtol=1e-6, atol=1e-7)
        assert torch.allclose(m2[lo:hi], v_, rtol=1e-6, atol=1e-9)
    assert abs(float(clip) - c) < 1e-5
    assert torch.equal(pg.param()[4096:8192], master.to(torch.bfloat16))


def _step_cfg(parallelism):  # noqa: ANN001, ANN202
    from priml_b200.loss import TokenCrossEntropy
    from priml_b200.models.presets import dense_lm
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.train import TrainStep

    return TrainStep.Config(
        model=dense_lm(vocab=1024, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
                       rope_theta=5e5),  # fmt: skip
        optimizer=FusedAdamW.Config(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1),
        loss=TokenCrossEntropy.Config(),
        parallelism=parallelism,
        dtype_autocast=torch.bfloat16,
        gradient_clip_norm=1.0,
    )


def _losses(parallelism, world: int = 1, rank: int = 0, steps: int = 4) -> list[float]:  # noqa: ANN001
    torch.manual_seed(0)
    step = _step_cfg(parallelism).make()
    g = torch.Generator(device="cuda").manual_seed(0)
    out = []
    for _ in range(steps):
        seq = torch.randint(0, 1024, (4, 257), device="cuda", generator=g)
        local = seq.chunk(world)[rank]
        o = step.train_step(tokens=local[:, :-1], targets=local[:, 1:])
        t = o["loss"].detach().float().mean()
        if world > 1:
            torch.distributed.all_reduce(t)
        out.append(float(t) / world)
    torch.cuda.synchronize()
    assert int(_native().read_status(True)) == 0
    return out


def test_fused_sharded_train_step_single_gpu_tracks_unsharded() -> None:
    from priml_b200.parallel.fused_fsdp import FusedFullySharded
    from priml_b200.parallel.strategies import NoParallel

    fused = _losses(FusedFullySharded.Config())
    plain = _losses(NoParallel.Config())
    for a, b in zip(fused, plain, strict=True):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), (fused, plain)
    assert all(x == x and 0.0 < x < 20.0 for x in fused)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q, shard_params: bool = False) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))  # fmt: skip
    torch.cuda.set_device(rank)
    import datetime

    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                         device_id=torch.device("cuda", rank))  # fmt: skip
    try:
        from priml_b200.parallel.fused_fsdp import FusedFullySharded

        q.put((rank, _losses(FusedFullySharded.Config(timeout_s=30.0, shard_params=shard_params), world, rank)))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_sharded_two_gpus_matches_one() -> None:
    import torch.multiprocessing as mp

    from priml_b200.parallel.fused_fsdp import FusedFullySharded

    one = _losses(FusedFullySharded.Config())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert isinstance(res[0], list), res
    assert res[0] == res[1]
    for a, b in zip(res[0], one, strict=True):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), (res[0], one)


def _run_two(shard_params: bool) -> dict:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, shard_params)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_weights_two_gpus_match_resident_weights() -> None:
    """1/R bf16 weights per rank, blocks gathered by the copy engines a block ahead: the same losses,
    bit for bit, as resident weights (the same bf16 values reach the same kernels)."""
    resident = _run_two(False)
    sharded = _run_two(True)
    assert isinstance(sharded[0], list), sharded
    assert sharded[0] == sharded[1]
    assert sharded[0] == resident[0], (sharded[0], resident[0])


def test_sharded_weights_single_gpu_matches_resident() -> None:
    from priml_b200.parallel.fused_fsdp import FusedFullySharded

    assert _losses(FusedFullySharded.Config(shard_params=True)) == _losses(FusedFullySharded.Config())
