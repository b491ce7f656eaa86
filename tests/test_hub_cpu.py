"""HF-format checkpoints: a tiny random Qwen3 written as config.json + safetensors
loads into Qwen3 and matches transformers' own forward (eager attention)."""

from __future__ import annotations

import json

import pytest
import torch


def test_qwen3_hf_roundtrip_and_parity(tmp_path) -> None:  # noqa: ANN001
    transformers = pytest.importorskip("transformers")
    from safetensors.torch import save_file

    from priml_b200.models.qwen3 import Qwen3

    cfg = {
        "model_type": "qwen3", "vocab_size": 96, "hidden_size": 32, "intermediate_size": 64,
        "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16,
        "rms_norm_eps": 1e-6, "rope_theta": 10000.0, "tie_word_embeddings": False, "torch_dtype": "float32",
        "max_position_embeddings": 128, "hidden_act": "silu",
    }  # fmt: skip
    torch.manual_seed(0)
    hf_model = transformers.Qwen3ForCausalLM(transformers.Qwen3Config(**cfg, attn_implementation="eager")).eval()
    with torch.no_grad():
        for p in hf_model.parameters():
            p.normal_(0, 0.1)
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    save_file({k: v.contiguous() for k, v in hf_model.state_dict().items()}, str(tmp_path / "model.safetensors"))
    ours = Qwen3.load(tmp_path, hf_split_projections=True).eval()
    x = torch.randint(0, 96, (2, 11))
    with torch.no_grad():
        ref = hf_model(x).logits
        got = ours(x)
    assert torch.allclose(got, ref, atol=1e-4), float((got - ref).abs().max())
