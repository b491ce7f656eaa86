"""Failure detection on the device: a peer wait that runs out reports through the status word.

Every wait in this repository's kernels is bounded. When a peer never raises the
flag a kernel waits for, the kernel records ``kTimeoutPeer`` in the per-device
status word and returns; the host reads the code, and the CUDA context stays
usable. The test makes a wait run out on one GPU without any fault: a one-rank
peer group waits at its completion barrier for an epoch that nothing will ever
publish, with a half-second limit.
"""

from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

K_TIMEOUT_PEER = 5  # pb::kTimeoutPeer in ops/csrc/common.cuh


def test_peer_wait_times_out_reports_status_and_leaves_the_context_usable() -> None:
    from priml_b200 import ops
    from priml_b200.ops import native

    n = native()
    n.read_status(True)  # start from a clean status word
    group = n.PeerGroup(0, 1, 64, 64)
    group.open([group.handles()])

    t0 = time.perf_counter()
    group.barrier(1, 0.5)  # epoch 1 is never published: the bounded wait must give up
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert n.read_status(True) == K_TIMEOUT_PEER
    assert 0.4 < waited < 30.0

    # A wait that is already satisfied returns at once and leaves the status clean.
    group.barrier(0, 0.5)
    torch.cuda.synchronize()
    assert n.read_status(True) == 0

    # Ordinary kernels still run correctly on the same context.
    a = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(384, 512, device="cuda", dtype=torch.bfloat16)
    out = ops.linear(a, w)
    ref = a.float() @ w.float().T
    assert float((out.float() - ref).abs().max() / ref.abs().max()) < 2e-2
    assert n.read_status(True) == 0
    del group
