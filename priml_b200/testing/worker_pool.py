"""Multi-rank execution without a cluster (``priml/distributed/testing.py:40-406``).

``run_ranks(fn, world_size)`` spawns ``world_size`` CPU processes that join a
gloo process group on a fresh loopback port, build a ``DeviceMesh`` of the
requested shape, run ``fn(rank, world_size, *args)`` and return every rank's
result (or raise with every failing rank's traceback). ``WorkerPool`` keeps the
ranks alive between calls and dispatches pickled functions to them, with
rendezvous / dispatch timeouts and a bounded join-then-kill on shutdown.
"""

from __future__ import annotations

import os
import pickle
import socket
import traceback
from collections.abc import Callable
from typing import Any

import torch.multiprocessing as mp

__all__ = ["WorkerPool", "free_port", "run_ranks"]

_TIMEOUT_S = 60.0


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _init(rank: int, world: int, port: int, mesh_shape: dict[str, int] | None, timeout_s: float) -> None:
    import datetime

    import torch.distributed as dist

    os.environ.update(
        {"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank), "WORLD_SIZE": str(world),
         "LOCAL_RANK": str(rank)}  # fmt: skip
    )
    os.environ.setdefault("OMP_NUM_THREADS", "2")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    if mesh_shape:
        from priml_b200.parallel import runtime

        runtime.initialize_global_device_mesh(
            device=__import__("torch").device("cpu"), mesh_topology=mesh_shape, backend="gloo"
        )


def _entry(rank: int, world: int, port: int, fn: bytes, args: bytes, mesh: Any, out: Any, timeout_s: float) -> None:
    import torch.distributed as dist

    try:
        _init(rank, world, port, mesh, timeout_s)
        res = pickle.loads(fn)(rank, world, *pickle.loads(args))
        out.put((rank, True, pickle.dumps(res)))
    except BaseException:  # noqa: BLE001 -- report every failure to the parent
        out.put((rank, False, traceback.format_exc()))
    finally:
        try:
            from priml_b200.parallel import runtime

            runtime.destroy_global_device_mesh()
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def run_ranks(
    fn: Callable[..., Any],
    world_size: int,
    *args: Any,
    mesh_shape: dict[str, int] | None = None,
    timeout_s: float = _TIMEOUT_S,
) -> list[Any]:
    """Run ``fn(rank, world_size, *args)`` on ``world_size`` gloo ranks; return the results in rank order."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = free_port()
    procs = [
        ctx.Process(target=_entry, args=(r, world_size, port, pickle.dumps(fn), pickle.dumps(args), mesh_shape, out,
                                         timeout_s))  # fmt: skip
        for r in range(world_size)
    ]
    for p in procs:
        p.start()
    results: dict[int, Any] = {}
    errors: list[str] = []
    try:
        for _ in range(world_size):
            rank, ok, payload = out.get(timeout=timeout_s * 2)
            if ok:
                results[rank] = pickle.loads(payload)
            else:
                errors.append(f"rank {rank}:\n{payload}")
    except Exception as exc:  # noqa: BLE001 -- queue timeout: a rank hung or died
        errors.append(f"timed out waiting for ranks: {exc!r}")
    finally:
        for p in procs:
            p.join(timeout=10)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=5)
    if errors:
        raise RuntimeError("distributed run failed:\n" + "\n".join(errors))
    return [results[r] for r in range(world_size)]


def _pool_worker(rank: int, world: int, port: int, mesh: Any, inbox: Any, outbox: Any, timeout_s: float) -> None:
    try:
        _init(rank, world, port, mesh, timeout_s)
    except BaseException:  # noqa: BLE001
        outbox.put((rank, False, traceback.format_exc()))
        return
    outbox.put((rank, True, b"ready"))
    while True:
        msg = inbox.get()
        if msg is None:
            break
        fn, args = msg
        try:
            res = pickle.loads(fn)(rank, world, *pickle.loads(args))
            outbox.put((rank, True, pickle.dumps(res)))
        except BaseException:  # noqa: BLE001
            outbox.put((rank, False, traceback.format_exc()))
    try:
        import torch.distributed as dist

        from priml_b200.parallel import runtime

        runtime.destroy_global_device_mesh()
        if dist.is_initialized():
            dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


class WorkerPool:
    """Long-lived gloo ranks; ``pool(fn, *args)`` runs ``fn(rank, world, *args)`` on all of them."""

    def __init__(self, world_size: int, mesh_shape: dict[str, int] | None = None, timeout_s: float = _TIMEOUT_S):
        self.world_size = world_size
        self.mesh_shape = mesh_shape
        self.timeout_s = timeout_s
        self._spawn()

    def _spawn(self) -> None:
        ctx = mp.get_context("spawn")
        self.outbox = ctx.Queue()
        self.inboxes = [ctx.Queue() for _ in range(self.world_size)]
        port = free_port()
        self.procs = [
            ctx.Process(target=_pool_worker, args=(r, self.world_size, port, self.mesh_shape, self.inboxes[r],
                                                   self.outbox, self.timeout_s), daemon=True)  # fmt: skip
            for r in range(self.world_size)
        ]
        for p in self.procs:
            p.start()
        self._collect("rendezvous")

    def _collect(self, what: str) -> list[Any]:
        results: dict[int, Any] = {}
        errors = []
        for _ in range(self.world_size):
            try:
                rank, ok, payload = self.outbox.get(timeout=self.timeout_s * 2)
            except Exception as exc:  # noqa: BLE001
                self.close()
                raise RuntimeError(f"{what}: timed out waiting for a rank ({exc!r})") from exc
            if ok:
                results[rank] = payload
            else:
                errors.append(f"rank {rank}:\n{payload}")
        if errors:
            raise RuntimeError(f"{what} failed:\n" + "\n".join(errors))
        return [results[r] for r in range(self.world_size)]

    def __call__(self, fn: Callable[..., Any], *args: Any) -> list[Any]:
        dead = [r for r, p in enumerate(self.procs) if not p.is_alive()]
        if dead:
            self.close()
            self._spawn()
        msg = (pickle.dumps(fn), pickle.dumps(args))
        for q in self.inboxes:
            q.put(msg)
        return [pickle.loads(x) for x in self._collect("dispatch")]

    def close(self) -> None:
        for q in self.inboxes:
            try:
                q.put(None)
            except Exception:  # noqa: BLE001
                pass
        for p in self.procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
                p.join(timeout=5)

    def __enter__(self) -> WorkerPool:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()
