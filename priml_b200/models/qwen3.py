"""Qwen3 dense decoder (``priml/model/qwen3.py:50-276``).

``Qwen3.Config.from_hf(config_json)`` maps HF fields; ``Qwen3.load(path)``
builds the model and loads HF weights through :func:`remap_hf_state_dict`:
``q/k/v_proj`` -> ``proj_qkv [q + 2 kv, head_dim, hidden]`` and
``gate/up_proj`` -> ``up_proj [2 * inter, hidden]`` (gate rows first).
"""

from __future__ import annotations

from dataclasses import KW_ONLY
from pathlib import Path
from typing import Any

import torch
from torch import Tensor

from priml_b200.config import Makes
from priml_b200.models.attention import SelfAttention
from priml_b200.models.causal_lm import CausalLM
from priml_b200.models.norm import RMSNorm
from priml_b200.models.rope import RoPE
from priml_b200.models.swiglu import SwiGLU
from priml_b200.models.transformer import TransformerBlock

__all__ = ["Qwen3", "remap_hf_state_dict"]


class Qwen3(CausalLM):
    class Config(Makes["Qwen3"], CausalLM.Config, kw_only=False):
        vocab_size: int = -1
        _: KW_ONLY
        hidden_size: int = -1
        intermediate_size: int = -1
        num_hidden_layers: int = -1
        num_attention_heads: int = -1
        num_key_value_heads: int = -1
        head_dim: int = -1
        rms_norm_eps: float = 1e-6
        rope_theta: float = 1_000_000.0
        hf_inv_freq: bool = True
        hf_split_projections: bool = False

        @classmethod
        def from_hf(cls, config: dict[str, Any]) -> Qwen3.Config:
            if config.get("model_type") != "qwen3":
                raise ValueError(f"Expected model_type='qwen3', got {config.get('model_type')!r}.")
            theta = config.get("rope_theta")
            if theta is None:
                theta = (config.get("rope_parameters") or {}).get("rope_theta")
            h, n = int(config["hidden_size"]), int(config["num_attention_heads"])
            return cls(
                vocab_size=int(config["vocab_size"]),
                hidden_size=h,
                intermediate_size=int(config["intermediate_size"]),
                num_hidden_layers=int(config["num_hidden_layers"]),
                num_attention_heads=n,
                num_key_value_heads=int(config.get("num_key_value_heads") or n),
                head_dim=int(config.get("head_dim") or h // n),
                rms_norm_eps=float(config.get("rms_norm_eps", 1e-6)),
                rope_theta=float(theta if theta is not None else 1e6),
                tie_embeddings=bool(config.get("tie_word_embeddings", False)),
            )

        def finalize(self):  # noqa: ANN201
            if self.hidden_size < 1:
                raise ValueError(f"hidden_size must be > 0, got {self.hidden_size}.")
            if self.num_attention_heads < 1:
                raise ValueError(f"num_attention_heads must be > 0, got {self.num_attention_heads}.")
            if self.num_key_value_heads == -1:
                self.num_key_value_heads = self.num_attention_heads
            if self.head_dim == -1:
                self.head_dim = self.hidden_size // self.num_attention_heads
            self.channels = self.hidden_size
            self.num_layers = self.num_hidden_layers
            eps = self.rms_norm_eps
            self.block = TransformerBlock.Config(
                channels_in=self.hidden_size,
                attn=SelfAttention.Config(
                    channels_in=self.hidden_size,
                    heads=self.num_attention_heads,
                    channels_head=self.head_dim,
                    num_heads_kv=self.num_key_value_heads,
                    causal=True,
                    rope=RoPE.Config(self.head_dim, base=self.rope_theta, hf_inv_freq=self.hf_inv_freq),
                    norm_qk=RMSNorm.Config(eps=eps, elementwise_affine=True),
                    share_qk_norm=False,
                    split_qkv_projection=self.hf_split_projections,
                ),
                ffn=SwiGLU.Config(channels_in=self.hidden_size, channels_hidden=self.intermediate_size,
                                  split_gate_projection=self.hf_split_projections),  # fmt: skip
                norm1=RMSNorm.Config(eps=eps, elementwise_affine=True),
                norm2=RMSNorm.Config(eps=eps, elementwise_affine=True),
            )
            self.final_norm = RMSNorm.Config(eps=eps, elementwise_affine=True)
            return super().finalize()

    @classmethod
    def load(cls, path_or_repo: str | Path, *, device: torch.device | str | None = None,
             dtype: torch.dtype | None = None, **overrides: Any) -> Qwen3:  # fmt: skip
        from priml_b200.hub import load_config, load_local_state_dict, resolve_hf_dtype

        hf = load_config(path_or_repo)
        cfg = cls.Config.from_hf(hf)
        for k, v in overrides.items():
            setattr(cfg, k, v)
        model = cfg.make()
        sd = remap_hf_state_dict(load_local_state_dict(path_or_repo), cfg.copy_tree().finalize())
        model.load_state_dict(sd, strict=True)
        return model.to(device=device or "cpu", dtype=resolve_hf_dtype(hf, dtype))


def remap_hf_state_dict(hf_sd: dict[str, Tensor], config: Qwen3.Config) -> dict[str, Tensor]:
    """HF Qwen3 names -> this layout (pure transform)."""
    h, nq, nkv, d = config.hidden_size, config.num_attention_heads, config.num_key_value_heads, config.head_dim
    out = {"embed.weight": hf_sd["model.embed_tokens.weight"], "final_norm.weight": hf_sd["model.norm.weight"]}
    if not config.tie_embeddings:
        out["lm_head.weight"] = hf_sd["lm_head.weight"]
    for i in range(config.num_hidden_layers):
        p, b = f"model.layers.{i}", f"blocks.{i}"
        out[f"{b}.norm1.weight"] = hf_sd[f"{p}.input_layernorm.weight"]
        out[f"{b}.norm2.weight"] = hf_sd[f"{p}.post_attention_layernorm.weight"]
        q = hf_sd[f"{p}.self_attn.q_proj.weight"].view(nq, d, h)
        k = hf_sd[f"{p}.self_attn.k_proj.weight"].view(nkv, d, h)
        v = hf_sd[f"{p}.self_attn.v_proj.weight"].view(nkv, d, h)
        out[f"{b}.attn.proj_qkv.weight"] = torch.cat([q, k, v], dim=0)
        out[f"{b}.attn.proj_out.weight"] = hf_sd[f"{p}.self_attn.o_proj.weight"]
        out[f"{b}.attn.norm_q.weight"] = hf_sd[f"{p}.self_attn.q_norm.weight"]
        out[f"{b}.attn.norm_k.weight"] = hf_sd[f"{p}.self_attn.k_norm.weight"]
        out[f"{b}.ffn.up_proj.weight"] = torch.cat(
            [hf_sd[f"{p}.mlp.gate_proj.weight"], hf_sd[f"{p}.mlp.up_proj.weight"]], dim=0
        )
        out[f"{b}.ffn.down_proj.weight"] = hf_sd[f"{p}.mlp.down_proj.weight"]
    return out
