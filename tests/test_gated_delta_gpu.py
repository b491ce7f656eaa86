"""Gated delta-rule chunk scan kernels (``gdn_fwd`` / ``gdn_bwd``) against fp32 PyTorch oracles."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def _inputs(B: int, S: int, H: int, decay: float, seed: int = 0, grad: bool = False) -> tuple[torch.Tensor, ...]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    kw = {"device": "cuda", "generator": g}
    q = torch.randn(B, S, H, 128, **kw)
    k = torch.randn(B, S, H, 128, **kw)
    v = torch.randn(B, S, H, 128, **kw)
    lg = -torch.rand(B, S, H, **kw) * decay
    beta = torch.rand(B, S, H, **kw)
    out = (q, k, v, lg, beta)
    return tuple(t.requires_grad_() for t in out) if grad else out


@pytest.mark.parametrize("B,S,H,decay", [(1, 128, 1, 0.5), (2, 300, 3, 0.5), (2, 2048, 4, 0.1), (1, 1000, 2, 20.0)])
def test_scan_kernels_match_torch_scan(B: int, S: int, H: int, decay: float) -> None:
    """The kernels against the same scan in fp32 on the same bf16 operands (state rounding only)."""
    from priml_b200.ops import native
    from priml_b200.ops.gated_delta import chunk_operands, scan_reference, scan_reference_bwd

    w, ut, qg, mqk, kr, gc = chunk_operands(*_inputs(B, S, H, decay))
    w, qg, mqk, kr = (x.to(torch.bfloat16).contiguous() for x in (w, qg, mqk, kr))
    ut, gc = ut.contiguous(), gc.contiguous()
    o, hs, us = native().gdn_fwd(w, ut, qg, mqk, kr, gc)
    o_ref, hs_ref, us_ref = scan_reference(w, ut, qg, mqk, kr, gc)
    assert _rel(o, o_ref) < 2e-2
    assert _rel(hs, hs_ref) < 2e-2
    assert _rel(us, us_ref) < 2e-2
    do = torch.randn(o.shape, device="cuda").to(torch.bfloat16)
    du, dhs = native().gdn_bwd(kr, mqk, do, qg, w, gc)
    du_ref, dhs_ref = scan_reference_bwd(kr, mqk, do, qg, w, gc)
    assert _rel(du, du_ref) < 2e-2
    assert _rel(dhs, dhs_ref) < 2e-2
    assert native().read_status() == 0


@pytest.mark.parametrize("S,decay", [(300, 0.5), (256, 20.0)])
def test_gated_delta_rule_matches_recurrence(S: int, decay: float) -> None:
    """Output and input gradients of the whole op against the token-by-token fp32 recurrence."""
    from priml_b200.models.gated_delta_net import gated_delta_recurrent
    from priml_b200.ops.gated_delta import gated_delta_rule

    q, k, v, lg, beta = _inputs(2, S, 2, decay, grad=True)
    out = gated_delta_rule(q, k, v, lg, beta)
    ref = gated_delta_recurrent(q, k, v, lg, beta)
    assert _rel(out, ref) < 2e-2
    do = torch.randn_like(ref)
    grads = torch.autograd.grad(out, (q, k, v, lg, beta), do)
    refs = torch.autograd.grad(ref, (q, k, v, lg, beta), do)
    for name, a, b in zip("q k v g beta".split(), grads, refs):
        assert _rel(a, b) < 3e-2, name


def test_gated_delta_net_module_cuda_matches_cpu() -> None:
    """The module on CUDA (kernel path) against the same weights on CPU (torch chunked path)."""
    from priml_b200.models.gated_delta_net import GatedDeltaNet

    torch.manual_seed(0)
    net = GatedDeltaNet.Config(256, heads_k=2, heads_v=4, channels_k_head=128, channels_v_head=128).make()
    x = torch.randn(2, 333, 256)
    xc = x.clone().requires_grad_()
    y_cpu = net(xc)
    y_cpu.square().mean().backward()
    net_gpu = GatedDeltaNet.Config(256, heads_k=2, heads_v=4, channels_k_head=128, channels_v_head=128).make()
    net_gpu.load_state_dict(net.state_dict())
    net_gpu.cuda()
    xg = x.cuda().requires_grad_()
    y = net_gpu(xg)
    y.square().mean().backward()
    assert _rel(y.cpu(), y_cpu) < 3e-2
    assert _rel(xg.grad.cpu(), xc.grad) < 5e-2
    for (name, p), (_, pc) in zip(net_gpu.named_parameters(), net.named_parameters()):
        assert _rel(p.grad.cpu(), pc.grad) < 5e-2, name
