"""This framework's modules against the reference's golden files and its own modules.

The reference ships bit-for-bit goldens (``*/goldens/*_min_cpu.pt``: a module's
state dict, an input and the output of its CPU forward) for five model blocks and
for the nanochat (including the model its experiment ladder builds), CIFAR-10 and
sudoku models. Each case builds the module here
with the golden test's configuration, loads the reference state dict strictly (so
parameter names and shapes are the reference's) and checks:

* the forward against the stored output, to fp32 rounding. Exact bits are not
  asserted there: the goldens were minted under the reference's math-library
  settings (``MKL_CBWR``, thread caps), which order fp32 reductions differently;
* the forward against the reference's own module, built from the same
  configuration in this process: bitwise equal (for the CIFAR-10 networks the
  batch-norm running statistics after the forward too), except where this
  framework evaluates in another order by design -- the MoE (one grouped pass over
  padded expert segments instead of a loop over experts), the gated delta rule
  (its own chunked derivation) and the MMDiT block (streams concatenated once) --
  which must agree to fp32 rounding.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any

import pytest
import torch
from torch import nn

from priml_b200.testing.reference import REFERENCE_ROOT, load_reference

pytestmark = pytest.mark.skipif(not (REFERENCE_ROOT / "priml").is_dir(), reason="the reference copy is not present")


def _golden(rel: str) -> dict[str, Any]:
    return torch.load(REFERENCE_ROOT / "priml" / rel, weights_only=True)


def _out(result: Any) -> torch.Tensor:
    if hasattr(result, "logits"):
        return result.logits
    return result[0] if isinstance(result, (tuple, list)) else result


# ---------------------------------------------------------------- the two sides of every case
def _moe(ref: bool) -> nn.Module:
    if ref:
        from priml.model.moe import MoE, Router
    else:
        from priml_b200.models.moe import MoE, Router
    return MoE.Config(channels_in=16, router=Router.Config(num_experts=4, top_k=2)).make()


def _mla(ref: bool) -> nn.Module:
    if ref:
        from priml.model.mla import MultiHeadLatentAttention
        from priml.model.rope import RoPE
    else:
        from priml_b200.models.mla import MultiHeadLatentAttention
        from priml_b200.models.rope import RoPE
    return MultiHeadLatentAttention.Config(channels_in=16, heads=2, channels_qk_nope_head=8, channels_qk_rope_head=4,
                                           channels_v_head=8, kv_lora_rank=8,
                                           rope=RoPE.Config(channels_head=4, base=10_000)).make()  # fmt: skip


def _gated_delta(ref: bool) -> nn.Module:
    if ref:
        from priml.model.gated_delta_net import GatedDeltaNet
    else:
        from priml_b200.models.gated_delta_net import GatedDeltaNet
    return GatedDeltaNet.Config(channels_in=16, heads_k=2, heads_v=2, channels_k_head=8, channels_v_head=8).make()


def _mmdit(ref: bool) -> nn.Module:
    if ref:
        from priml.model.attention import MultiStreamAttention
        from priml.model.mmdit import MMDiTBlock
    else:
        from priml_b200.models.attention import MultiStreamAttention
        from priml_b200.models.vision import MMDiTBlock
    cfg = MMDiTBlock.Config(channels_in=16, num_streams=2)
    cfg.attn = MultiStreamAttention.Config(heads=2)
    return cfg.make()


def _block(ref: bool) -> nn.Module:
    if ref:
        from priml.model.attention import SelfAttention
        from priml.model.transformer import TransformerBlock
    else:
        from priml_b200.models.attention import SelfAttention
        from priml_b200.models.transformer import TransformerBlock
    return TransformerBlock.Config(channels_in=16, attn=SelfAttention.Config(heads=2, channels_head=8)).make()


def _nanochat(ref: bool, **overrides: Any) -> nn.Module:
    if ref:
        from priml.baselines.nanochat.model import NanoChatLM
    else:
        from priml_b200.baselines.nanochat.model import NanoChatLM
    cfg = NanoChatLM.Config()
    cfg.vocab_size, cfg.max_seq_len, cfg.channels_in, cfg.num_layers = 32, 16, 16, 2
    cfg.template.attn.window_pattern = "L"
    cfg.template.attn.channels_head = 8
    cfg.template.attn.gate_channels = 4
    for name, value in overrides.items():
        setattr(cfg, name, value)
    return cfg.make()


def _resnet(ref: bool) -> nn.Module:
    if ref:
        from priml.baselines.cifar10.model import ResNet
    else:
        from priml_b200.baselines.cifar10.model import ResNet
    cfg = ResNet.Config()
    cfg.channels_hidden = (8, 16)
    cfg.blocks_per_stage = 1
    return cfg.make()


def _speednet(ref: bool) -> nn.Module:
    if ref:
        from priml.baselines.cifar10.model import ConvBlock, SpeedNet
    else:
        from priml_b200.baselines.cifar10.model import ConvBlock, SpeedNet
    cfg = SpeedNet.Config()
    cfg.channels_hidden = (8, 16, 24)
    cfg.block = ConvBlock.Config()
    cfg.block.num_convs = 1
    return cfg.make()


def _sudoku(ref: bool, recurrent: bool = False) -> nn.Module:
    if ref:
        from priml.baselines.sudoku.model import DeepRecurrence, GridEmbedding, SudokuNet
        from priml.model.swiglu import SwiGLU
        from priml.model.transformer import TransformerBlock
    else:
        from priml_b200.baselines.sudoku.model import DeepRecurrence, GridEmbedding, SudokuNet
        from priml_b200.models.swiglu import SwiGLU
        from priml_b200.models.transformer import TransformerBlock
    cfg = SudokuNet.Config(hidden_size=16, num_layers=1)
    cfg.embedding = GridEmbedding.Config()
    cfg.block = TransformerBlock.Config(prenorm=False, ffn=SwiGLU.Config(round_to=16))
    if recurrent:
        cfg.recurrence = DeepRecurrence.Config(slow_cycles=2, fast_cycles=2)
    return cfg.make()


def _nanochat_smoke(ref: bool) -> nn.Module:
    """The model the experiment ladder's smallest rung builds (exp_smoke, run under bf16 autocast)."""
    if ref:
        from priml.baselines.nanochat import experiments
    else:
        from priml_b200.baselines.nanochat import experiments
    return experiments.exp_smoke().step.model.make()


# cases evaluated in another order than the reference's module (see the module docstring)
REORDERED = {"moe", "gated_delta_net", "mmdit_block"}

# golden file, builder, tolerance against the stored output (relative to its largest entry)
CASES: dict[str, tuple[str, Callable[..., nn.Module], float]] = {
    "moe": ("model/goldens/moe_min_cpu.pt", _moe, 1e-5),
    "mla": ("model/goldens/mla_min_cpu.pt", _mla, 1e-5),
    "gated_delta_net": ("model/goldens/gated_delta_net_min_cpu.pt", _gated_delta, 1e-5),
    "mmdit_block": ("model/goldens/mmdit_block_min_cpu.pt", _mmdit, 1e-5),
    "transformer_block": ("model/goldens/transformer_block_min_cpu.pt", _block, 1e-5),
    "nanochat": ("baselines/nanochat/goldens/plain_min_cpu.pt", _nanochat, 1e-5),
    "nanochat_value_embedding": ("baselines/nanochat/goldens/value_embedding_min_cpu.pt",
                                 lambda ref: _nanochat(ref, value_embedding_stride=1), 1e-5),  # fmt: skip
    # bf16 autocast: the mint host's bf16 matmuls round differently from this host's
    "nanochat_exp_smoke": ("baselines/nanochat/goldens/exp_smoke_forward_min_cpu.pt", _nanochat_smoke, 3e-2),
    "cifar10_resnet": ("baselines/cifar10/goldens/resnet_min_cpu.pt", _resnet, 1e-5),
    "cifar10_speednet": ("baselines/cifar10/goldens/speednet_min_cpu.pt", _speednet, 1e-5),
    # the post-norm recurrence compounds the reduction-order difference over its cycles
    "sudoku": ("baselines/sudoku/goldens/plain_min_cpu.pt", _sudoku, 1e-4),
    "sudoku_recurrent": ("baselines/sudoku/goldens/recurrent_min_cpu.pt", lambda ref: _sudoku(ref, True), 1e-3),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_module_matches_reference_golden_and_module(name: str) -> None:
    load_reference()
    path, build, tol = CASES[name]
    golden = _golden(path)
    ours, theirs = build(False), build(True)
    ours.load_state_dict(golden["state_dict"], strict=True)
    theirs.load_state_dict(golden["state_dict"], strict=True)
    autocast = torch.amp.autocast(device_type="cpu", dtype=torch.bfloat16, enabled=name == "nanochat_exp_smoke")
    with torch.no_grad(), autocast:
        out = _out(ours(golden["input"]))
        ref_out = _out(theirs(golden["input"]))
    stored = golden["output"]
    assert out.shape == stored.shape and out.dtype == stored.dtype
    err = float((out - stored).abs().max() / stored.abs().max())
    assert err < tol, err
    if name in REORDERED:
        assert float((out - ref_out).abs().max() / ref_out.abs().max()) < 1e-5
    else:
        assert torch.equal(out, ref_out), float((out - ref_out).abs().max())
    ref_state = theirs.state_dict()
    for key, value in ours.state_dict().items():  # buffers a forward updates (batch-norm statistics)
        assert torch.equal(value, ref_state[key]), key
