"""This framework's blocks against the reference's own golden files.

The reference ships bit-for-bit goldens for five blocks
(``priml/model/goldens/*_min_cpu.pt``: the module's state dict, an input and the
output its CPU forward produced). Each block is built here with the golden
test's configuration (``priml/model/{moe,mla,gated_delta_net,mmdit,transformer}_golden_test.py``),
the reference state dict is loaded strictly (so the parameter names and shapes
are the reference's), and the forward must reproduce the stored output to fp32
rounding. Exact bits are not asserted: the goldens were minted under the
reference's math-library settings (``MKL_CBWR``, thread caps), which order the
fp32 reductions differently.
"""

from __future__ import annotations

from collections.abc import Callable

import pytest
import torch
from torch import nn

from priml_b200.testing.reference import REFERENCE_ROOT

GOLDENS = REFERENCE_ROOT / "priml" / "model" / "goldens"

pytestmark = pytest.mark.skipif(not GOLDENS.is_dir(), reason="the reference copy is not present")


def _moe() -> nn.Module:
    from priml_b200.models.moe import MoE, Router

    return MoE.Config(channels_in=16, router=Router.Config(num_experts=4, top_k=2)).make()


def _mla() -> nn.Module:
    from priml_b200.models.mla import MultiHeadLatentAttention
    from priml_b200.models.rope import RoPE

    return MultiHeadLatentAttention.Config(channels_in=16, heads=2, channels_qk_nope_head=8, channels_qk_rope_head=4,
                                           channels_v_head=8, kv_lora_rank=8,
                                           rope=RoPE.Config(channels_head=4, base=10_000)).make()  # fmt: skip


def _gated_delta() -> nn.Module:
    from priml_b200.models.gated_delta_net import GatedDeltaNet

    return GatedDeltaNet.Config(channels_in=16, heads_k=2, heads_v=2, channels_k_head=8, channels_v_head=8).make()


def _mmdit() -> nn.Module:
    from priml_b200.models.attention import MultiStreamAttention
    from priml_b200.models.vision import MMDiTBlock

    cfg = MMDiTBlock.Config(channels_in=16, num_streams=2)
    cfg.attn = MultiStreamAttention.Config(heads=2)
    return cfg.make()


def _block() -> nn.Module:
    from priml_b200.models.attention import SelfAttention
    from priml_b200.models.transformer import TransformerBlock

    return TransformerBlock.Config(channels_in=16, attn=SelfAttention.Config(heads=2, channels_head=8)).make()


CASES: dict[str, Callable[[], nn.Module]] = {
    "moe_min_cpu": _moe,
    "mla_min_cpu": _mla,
    "gated_delta_net_min_cpu": _gated_delta,
    "mmdit_block_min_cpu": _mmdit,
    "transformer_block_min_cpu": _block,
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_block_reproduces_reference_golden(name: str) -> None:
    golden = torch.load(GOLDENS / f"{name}.pt", weights_only=True)
    module = CASES[name]()
    module.load_state_dict(golden["state_dict"], strict=True)
    with torch.no_grad():
        out = module(golden["input"])
    out = out[0] if isinstance(out, (tuple, list)) else out
    ref = golden["output"]
    assert out.shape == ref.shape and out.dtype == ref.dtype
    err = float((out - ref).abs().max() / ref.abs().max())
    assert err < 1e-5, err
