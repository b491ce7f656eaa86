"""Padded device-side MoE dispatch and the grouped expert path (CPU reference kernels)."""

from __future__ import annotations

import torch

from priml_b200.ops.grouped import grouped_swiglu_experts, padded_dispatch_plan


def test_padded_plan_segments_are_aligned_and_stable() -> None:
    g = torch.Generator().manual_seed(0)
    idx = torch.randint(0, 5, (37, 3), generator=g)
    idx[:, 0] = torch.where(idx[:, 0] == 4, 3, idx[:, 0])  # expert 4 gets few rows
    pos, off, cap = padded_dispatch_plan(idx, 6)  # expert 5 gets none
    off = off.tolist()
    assert all(o % 128 == 0 for o in off) and off[-1] <= cap
    assert off[6] == off[5]  # empty expert: empty segment
    flat = idx.reshape(-1)
    assert len(set(pos.tolist())) == flat.numel()
    for e in range(6):
        slots = (flat == e).nonzero().flatten()
        rows = pos[slots]
        # slots of expert e fill its segment from the start, in slot order
        assert rows.tolist() == list(range(off[e], off[e] + len(slots)))


def test_grouped_experts_match_per_expert_loop() -> None:
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(1)
    t, k, e, c, h = 29, 2, 4, 16, 24
    x = torch.randn(t, c, generator=g, requires_grad=True)
    up = (torch.randn(e, 2 * h, c, generator=g) / c**0.5).requires_grad_()
    down = (torch.randn(e, c, h, generator=g) / h**0.5).requires_grad_()
    idx = torch.randint(0, e, (t, k), generator=g)
    w = torch.rand(t, k, generator=g)
    y = grouped_swiglu_experts(x, w, idx, up, down)
    want = torch.zeros(t, c)
    for ti in range(t):
        for j in range(k):
            ei = int(idx[ti, j])
            gate, u = F.linear(x[ti], up[ei]).chunk(2)
            want[ti] += w[ti, j] * F.linear(F.silu(gate) * u, down[ei])
    torch.testing.assert_close(y, want, rtol=1e-5, atol=1e-5)
    gy = torch.randn(t, c, generator=g)
    da = torch.autograd.grad(y, (x, up, down), gy)
    db = torch.autograd.grad(want, (x, up, down), gy)
    for a, b in zip(da, db, strict=True):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)


def test_moe_module_grouped_equals_loop_dispatch() -> None:
    from priml_b200.models.moe import MoE, Router
    from priml_b200.models.swiglu import SwiGLU

    torch.manual_seed(0)
    m = MoE.Config(channels_in=32, router=Router.Config(num_experts=4, top_k=2),
                   expert=SwiGLU.Config(channels_hidden=48)).make()  # fmt: skip
    x = torch.randn(2, 9, 32)
    weights, indices, _ = m.router(x.reshape(-1, 32))
    a = m._dispatch_grouped(x.reshape(-1, 32), weights, indices)  # noqa: SLF001
    # loop over experts with the same stacked weights
    want = torch.zeros(18, 32)
    for s in range(indices.numel()):
        ti, j = divmod(s, 2)
        ei = int(indices[ti, j])
        gu = x.reshape(-1, 32)[ti] @ m.experts.up_proj[ei].t()
        gate, up = gu.chunk(2)
        want[ti] += weights[ti, j] * ((torch.nn.functional.silu(gate) * up) @ m.experts.down_proj[ei].t())
    torch.testing.assert_close(a, want, rtol=1e-5, atol=1e-5)


def test_moe_built_on_meta_materializes_every_expert() -> None:
    from priml_b200.models.moe import MoE, Router
    from priml_b200.models.swiglu import SwiGLU
    from priml_b200.parallel.strategies import materialize_meta

    with torch.device("meta"):
        m = MoE.Config(channels_in=32, router=Router.Config(num_experts=4, top_k=2),
                       expert=SwiGLU.Config(channels_hidden=48)).make()  # fmt: skip
    assert m.experts.up_proj.is_meta
    m = materialize_meta(m, torch.device("cpu"))  # raises on any tensor left uninitialized
    assert not m.experts.up_proj.is_meta and float(m.experts.up_proj.std()) > 0
    assert not torch.equal(m.experts.up_proj[0], m.experts.up_proj[1])  # each expert drawn afresh
