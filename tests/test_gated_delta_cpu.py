"""Chunked gated delta rule (``priml_b200.ops.gated_delta``) against the token-by-token recurrence.

On CPU the chunk scan runs in its torch restatement (:func:`scan_reference` forward,
:func:`scan_reference_bwd` for the hand-derived backward), so these tests check the
algebra the CUDA kernels implement: the chunk-parallel operands, the scan, and the
gradients of the scan's inputs.
"""

from __future__ import annotations

import pytest
import torch

from priml_b200.models.gated_delta_net import GatedDeltaNet, gated_delta_recurrent
from priml_b200.ops.gated_delta import gated_delta_rule


def _inputs(B: int, S: int, H: int, d: int, decay: float, seed: int = 0) -> tuple[torch.Tensor, ...]:
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, H, d, generator=g, requires_grad=True)
    k = torch.randn(B, S, H, d, generator=g, requires_grad=True)
    v = torch.randn(B, S, H, d, generator=g, requires_grad=True)
    lg = (-torch.rand(B, S, H, generator=g) * decay).requires_grad_()
    beta = torch.rand(B, S, H, generator=g).requires_grad_()
    return q, k, v, lg, beta


@pytest.mark.parametrize("S,decay", [(128, 0.5), (300, 0.5), (300, 20.0), (256, 0.0)])
def test_chunk_scan_matches_recurrence(S: int, decay: float) -> None:
    q, k, v, lg, beta = _inputs(2, S, 2, 128, decay)
    out = gated_delta_rule(q, k, v, lg, beta)
    ref = gated_delta_recurrent(q, k, v, lg, beta)
    assert out.shape == ref.shape
    torch.testing.assert_close(out, ref, atol=2e-6, rtol=1e-4)
    do = torch.randn_like(out)
    grads = torch.autograd.grad((out * do).sum(), (q, k, v, lg, beta))
    refs = torch.autograd.grad((ref * do).sum(), (q, k, v, lg, beta))
    for name, a, b in zip("q k v g beta".split(), grads, refs):
        err = float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))
        assert err < 1e-4, f"d{name}: {err}"


def test_module_cpu_path_is_finite_under_strong_decay() -> None:
    torch.manual_seed(0)
    net = GatedDeltaNet.Config(256, heads_k=2, heads_v=4, channels_k_head=128, channels_v_head=128).make()
    x = torch.randn(2, 140, 256, requires_grad=True)
    y = net(x)
    y.square().mean().backward()
    assert torch.isfinite(y).all() and torch.isfinite(x.grad).all()
