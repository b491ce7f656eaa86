"""Pieces without a test of their own so far, checked against the reference's code where it has one.

* YaRN RoPE tables and the Kimi-K2 (MLA + MoE) HF checkpoint remap: the same
  inputs through the reference package and through this one give the same
  tables, the same remapped state dict, and the same model output.
* Layer activation checkpointing leaves the gradients unchanged.
* Trackers write what they are given; the cost model adds up.
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import pytest
import torch

from priml_b200.testing.reference import load_reference, reference_available

needs_reference = pytest.mark.skipif(not reference_available(), reason="the reference copy is not present")

YARN = {"type": "yarn", "factor": 32.0, "original_max_position_embeddings": 256, "beta_fast": 32.0,
        "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0}  # fmt: skip


@needs_reference
def test_yarn_rope_tables_match_reference() -> None:
    load_reference()
    from priml.model.rope import RoPE as RefRoPE
    from priml.model.rope import YarnScaling as RefYarn

    from priml_b200.models.rope import RoPE, YarnScaling

    fields = {k: v for k, v in YARN.items() if k != "type"}
    ref = RefRoPE.Config(64, base=1e4, yarn=RefYarn(**fields)).make()
    ours = RoPE.Config(64, base=1e4, yarn=YarnScaling(**fields)).make()
    pos = torch.arange(0, 9000, 7)
    for a, b in zip(ours(pos), ref(pos), strict=True):
        torch.testing.assert_close(a.float(), b.float(), rtol=1e-6, atol=1e-6)


def _kimi_hf_config() -> dict:
    return {"model_type": "kimi_k2", "vocab_size": 64, "hidden_size": 32, "num_hidden_layers": 3,
            "num_attention_heads": 4, "qk_nope_head_dim": 8, "qk_rope_head_dim": 8, "v_head_dim": 8,
            "q_lora_rank": None, "kv_lora_rank": 16, "intermediate_size": 48, "moe_intermediate_size": 16,
            "n_routed_experts": 4, "num_experts_per_tok": 2, "n_shared_experts": 1, "first_k_dense_replace": 1,
            "scoring_func": "sigmoid", "routed_scaling_factor": 2.5, "norm_topk_prob": True, "rms_norm_eps": 1e-6,
            "rope_theta": 1e4, "rope_scaling": YARN, "tie_word_embeddings": False}  # fmt: skip


def _kimi_hf_state_dict(cfg: dict) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(0)
    h, v = cfg["hidden_size"], cfg["vocab_size"]
    heads, nope, rope, vd = cfg["num_attention_heads"], cfg["qk_nope_head_dim"], cfg["qk_rope_head_dim"], cfg["v_head_dim"]
    kvr, inter, moe_i, n_exp = cfg["kv_lora_rank"], cfg["intermediate_size"], cfg["moe_intermediate_size"], cfg["n_routed_experts"]
    shapes = {"model.embed_tokens.weight": (v, h), "model.norm.weight": (h,), "lm_head.weight": (v, h)}
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        shapes |= {f"{p}.input_layernorm.weight": (h,), f"{p}.post_attention_layernorm.weight": (h,),
                   f"{p}.self_attn.q_proj.weight": (heads * (nope + rope), h),
                   f"{p}.self_attn.kv_a_proj_with_mqa.weight": (kvr + rope, h),
                   f"{p}.self_attn.kv_a_layernorm.weight": (kvr,),
                   f"{p}.self_attn.kv_b_proj.weight": (heads * (nope + vd), kvr),
                   f"{p}.self_attn.o_proj.weight": (h, heads * vd)}  # fmt: skip
        mlps = [(f"{p}.mlp", inter)] if i < cfg["first_k_dense_replace"] else (
            [(f"{p}.mlp.experts.{e}", moe_i) for e in range(n_exp)]
            + [(f"{p}.mlp.shared_experts", moe_i * cfg["n_shared_experts"])])  # fmt: skip
        for name, width in mlps:
            shapes |= {f"{name}.gate_proj.weight": (width, h), f"{name}.up_proj.weight": (width, h),
                       f"{name}.down_proj.weight": (h, width)}  # fmt: skip
        if i >= cfg["first_k_dense_replace"]:
            shapes |= {f"{p}.mlp.gate.weight": (n_exp, h), f"{p}.mlp.gate.e_score_correction_bias": (n_exp,)}
    out = {k: torch.randn(s, generator=g) * (0.02 if len(s) > 1 else 1.0) for k, s in shapes.items()}
    for k in out:  # norm weights near one
        if k.endswith("norm.weight") or k.endswith("layernorm.weight"):
            out[k] = 1.0 + 0.1 * out[k]
    return out


@needs_reference
def test_kimi_k2_remap_and_forward_match_reference() -> None:
    load_reference()
    from priml.model.kimi_k2 import KimiK2 as RefKimi
    from priml.model.kimi_k2 import remap_hf_state_dict as ref_remap

    from priml_b200.models.kimi_k2 import KimiK2, remap_hf_state_dict

    hf_cfg = _kimi_hf_config()
    hf_sd = _kimi_hf_state_dict(hf_cfg)
    ref_cfg, our_cfg = RefKimi.Config.from_hf(hf_cfg), KimiK2.Config.from_hf(hf_cfg)
    ref_sd, our_sd = ref_remap(hf_sd, ref_cfg), remap_hf_state_dict(hf_sd, our_cfg)
    assert sorted(ref_sd) == sorted(our_sd)
    for k in ref_sd:
        assert torch.equal(ref_sd[k], our_sd[k]), k
    ref_model, our_model = ref_cfg.make(), our_cfg.make()
    ref_model.load_state_dict(ref_sd)
    our_model.load_state_dict(our_sd)
    tokens = torch.randint(0, hf_cfg["vocab_size"], (2, 12), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        torch.testing.assert_close(our_model(tokens), ref_model(tokens), rtol=1e-5, atol=1e-5)


def test_layer_activation_checkpointing_keeps_gradients() -> None:
    from priml_b200.models.presets import tiny_lm
    from priml_b200.train.activation import LayerActivationCheckpointing

    torch.manual_seed(0)
    plain = tiny_lm().make()
    recomputed = tiny_lm().make()
    recomputed.load_state_dict(plain.state_dict())
    LayerActivationCheckpointing.Config().make()(recomputed)
    tokens = torch.randint(0, 512, (2, 32))
    for m in (plain, recomputed):
        m.token_loss(tokens[:, :-1], tokens[:, 1:]).mean().backward()
    for (name, a), (_, b) in zip(plain.named_parameters(), recomputed.named_parameters(), strict=True):
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-6, atol=1e-7, msg=name)


def test_trackers_record_metrics(tmp_path: Path) -> None:
    from priml_b200.train.tracker import AsyncTracker, FileTracker, TrackerList

    both = TrackerList.Config(trackers=[
        FileTracker.Config(path=str(tmp_path / "a.jsonl")),
        AsyncTracker.Config(inner=FileTracker.Config(path=str(tmp_path / "b.jsonl"))),  # written on a worker thread
    ]).make()  # fmt: skip
    for step in range(3):
        both.log({"loss": torch.tensor(2.0 - step), "lr": 1e-3}, step)
    both.flush()
    both.close()
    for name in ("a.jsonl", "b.jsonl"):
        rows = [json.loads(line) for line in (tmp_path / name).read_text().splitlines()]
        assert [r["step"] for r in rows] == [0, 1, 2]
        assert [r["loss"] for r in rows] == [2.0, 1.0, 0.0]
        assert all(r["lr"] == 1e-3 for r in rows)


def test_cost_model_flops_and_mfu() -> None:
    from priml_b200 import cost

    shape = cost.DenseLMShape(d_model=2048, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64, ffn_hidden=8192,
                              vocab=32768)  # fmt: skip
    per_layer = 2048 * (32 + 2 * 8) * 64 + 32 * 64 * 2048 + 3 * 2048 * 8192
    assert shape.matmul_params() == 16 * per_layer + 32768 * 2048
    fpt = cost.train_flops_per_token(shape, 4096)
    attn = cost.attention_flops(4096, 32, 64, 64, causal=True) * 16
    assert math.isclose(fpt, 6 * shape.matmul_params() + 3 * attn, rel_tol=1e-9)
    assert math.isclose(attn / 16, 2.0 * 4096 * 128 * 32 / 2, rel_tol=1e-12)  # causal: half of 2*S*(dqk+dv)*H
    peaks = cost.Peaks(hbm_gbs=6500.0, bf16_tflops=1600.0, bf16_tflops_sustained=1400.0, source="test")
    assert math.isclose(cost.mfu(1e5, fpt, 1, peaks, sustained=True), 1e5 * fpt / 1.4e15, rel_tol=1e-9)
