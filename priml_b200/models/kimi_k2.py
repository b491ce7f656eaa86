"""Kimi-K2 / DeepSeek-V3 decoder: MLA + first-k-dense + MoE (``priml/model/kimi_k2.py:69-445``)."""

from __future__ import annotations

from dataclasses import KW_ONLY
from pathlib import Path
from typing import Any, Literal

import torch
from torch import Tensor

from priml_b200.config import Makes
from priml_b200.models.causal_lm import CausalLM
from priml_b200.models.mla import MultiHeadLatentAttention
from priml_b200.models.moe import MoE, Router
from priml_b200.models.norm import RMSNorm
from priml_b200.models.rope import RoPE, YarnScaling
from priml_b200.models.swiglu import SwiGLU
from priml_b200.models.transformer import TransformerBlock

__all__ = ["KimiK2", "remap_hf_state_dict"]


class KimiK2(CausalLM):
    class Config(Makes["KimiK2"], CausalLM.Config, kw_only=False):
        vocab_size: int = -1
        _: KW_ONLY
        hidden_size: int = -1
        num_hidden_layers: int = -1
        num_attention_heads: int = -1
        channels_qk_nope_head: int = 128
        channels_qk_rope_head: int = 64
        channels_v_head: int = 128
        q_lora_rank: int | None = None
        kv_lora_rank: int = 512
        intermediate_size: int = -1
        moe_intermediate_size: int = -1
        n_routed_experts: int = 0
        num_experts_per_tok: int = 1
        n_shared_experts: int = 0
        first_k_dense_replace: int = 0
        n_group: int = 1
        topk_group: int = 1
        norm_topk_prob: bool = True
        routed_scaling_factor: float = 1.0
        scoring_func: Literal["softmax", "sigmoid"] = "sigmoid"
        rms_norm_eps: float = 1e-6
        rope_theta: float = 10_000.0
        yarn: YarnScaling | None = None

        @classmethod
        def from_hf(cls, config: dict[str, Any]) -> KimiK2.Config:
            rs = config.get("rope_scaling") or None
            yarn = None
            if rs and rs.get("type", rs.get("rope_type")) == "yarn":
                yarn = YarnScaling(
                    factor=float(rs["factor"]),
                    original_max_position_embeddings=int(rs["original_max_position_embeddings"]),
                    beta_fast=float(rs.get("beta_fast", 32.0)),
                    beta_slow=float(rs.get("beta_slow", 1.0)),
                    mscale=float(rs.get("mscale", 1.0)),
                    mscale_all_dim=float(rs.get("mscale_all_dim", 0.0)),
                )
            return cls(
                vocab_size=int(config["vocab_size"]),
                hidden_size=int(config["hidden_size"]),
                num_hidden_layers=int(config["num_hidden_layers"]),
                num_attention_heads=int(config["num_attention_heads"]),
                channels_qk_nope_head=int(config.get("qk_nope_head_dim", 128)),
                channels_qk_rope_head=int(config.get("qk_rope_head_dim", 64)),
                channels_v_head=int(config.get("v_head_dim", 128)),
                q_lora_rank=config.get("q_lora_rank"),
                kv_lora_rank=int(config.get("kv_lora_rank", 512)),
                intermediate_size=int(config["intermediate_size"]),
                moe_intermediate_size=int(config.get("moe_intermediate_size", -1)),
                n_routed_experts=int(config.get("n_routed_experts") or 0),
                num_experts_per_tok=int(config.get("num_experts_per_tok") or 1),
                n_shared_experts=int(config.get("n_shared_experts") or 0),
                first_k_dense_replace=int(config.get("first_k_dense_replace", 0)),
                n_group=int(config.get("n_group") or 1),
                topk_group=int(config.get("topk_group") or 1),
                norm_topk_prob=bool(config.get("norm_topk_prob", True)),
                routed_scaling_factor=float(config.get("routed_scaling_factor", 1.0)),
                scoring_func=config.get("scoring_func", "sigmoid"),
                rms_norm_eps=float(config.get("rms_norm_eps", 1e-6)),
                rope_theta=float(config.get("rope_theta", 10_000.0)),
                yarn=yarn,
                tie_embeddings=bool(config.get("tie_word_embeddings", False)),
            )

        def finalize(self):  # noqa: ANN201
            self.channels = self.hidden_size
            self.num_layers = self.num_hidden_layers
            eps = self.rms_norm_eps
            attn = MultiHeadLatentAttention.Config(
                channels_in=self.hidden_size,
                heads=self.num_attention_heads,
                channels_qk_nope_head=self.channels_qk_nope_head,
                channels_qk_rope_head=self.channels_qk_rope_head,
                channels_v_head=self.channels_v_head,
                q_lora_rank=self.q_lora_rank,
                kv_lora_rank=self.kv_lora_rank,
                rope=RoPE.Config(self.channels_qk_rope_head, base=self.rope_theta, yarn=self.yarn, hf_inv_freq=True),
            )
            # YaRN's attention-scale correction lives in the rotation tables (RoPE with ``yarn``
            # scales cos / sin), as in the reference; the softmax scale stays qk_head_dim ** -0.5.
            blocks = []
            for i in range(self.num_hidden_layers):
                if i < self.first_k_dense_replace or self.n_routed_experts == 0:
                    ffn: Any = SwiGLU.Config(channels_hidden=self.intermediate_size)
                else:
                    ffn = MoE.Config(
                        router=Router.Config(
                            num_experts=self.n_routed_experts, top_k=self.num_experts_per_tok,
                            scoring_func=self.scoring_func, norm_topk_prob=self.norm_topk_prob,
                            routed_scaling_factor=self.routed_scaling_factor, n_group=self.n_group,
                            topk_group=self.topk_group,
                        ),
                        expert=SwiGLU.Config(channels_hidden=self.moe_intermediate_size),
                        num_shared_experts=1 if self.n_shared_experts else 0,
                        shared_expert=SwiGLU.Config(channels_hidden=self.moe_intermediate_size * max(1, self.n_shared_experts)),
                    )  # fmt: skip
                blocks.append(TransformerBlock.Config(
                    channels_in=self.hidden_size, attn=attn.copy_tree(), ffn=ffn,
                    norm1=RMSNorm.Config(eps=eps, elementwise_affine=True),
                    norm2=RMSNorm.Config(eps=eps, elementwise_affine=True),
                ))  # fmt: skip
            self.block = blocks
            self.final_norm = RMSNorm.Config(eps=eps, elementwise_affine=True)
            return super().finalize()

    @classmethod
    def load(cls, path_or_repo: str | Path, *, device: torch.device | str | None = None,
             dtype: torch.dtype | None = None) -> KimiK2:  # fmt: skip
        from priml_b200.hub import load_config, load_local_state_dict, resolve_hf_dtype

        hf = load_config(path_or_repo)
        cfg = cls.Config.from_hf(hf)
        model = cfg.make()
        model.load_state_dict(remap_hf_state_dict(load_local_state_dict(path_or_repo), cfg.copy_tree().finalize()))
        return model.to(device=device or "cpu", dtype=resolve_hf_dtype(hf, dtype))


def _fused_mlp(hf_sd: dict[str, Tensor], src: str, dst: str, out: dict[str, Tensor]) -> None:
    out[f"{dst}.up_proj.weight"] = torch.cat([hf_sd[f"{src}.gate_proj.weight"], hf_sd[f"{src}.up_proj.weight"]], dim=0)
    out[f"{dst}.down_proj.weight"] = hf_sd[f"{src}.down_proj.weight"]


def remap_hf_state_dict(hf_sd: dict[str, Tensor], config: KimiK2.Config) -> dict[str, Tensor]:
    """HF Kimi-K2 / DeepSeek-V3 names -> this layout (per-expert keys, gate rows first)."""
    out = {"embed.weight": hf_sd["model.embed_tokens.weight"], "final_norm.weight": hf_sd["model.norm.weight"]}
    if not config.tie_embeddings:
        out["lm_head.weight"] = hf_sd["lm_head.weight"]
    for i in range(config.num_hidden_layers):
        p, b = f"model.layers.{i}", f"blocks.{i}"
        out[f"{b}.norm1.weight"] = hf_sd[f"{p}.input_layernorm.weight"]
        out[f"{b}.norm2.weight"] = hf_sd[f"{p}.post_attention_layernorm.weight"]
        a, ba = f"{p}.self_attn", f"{b}.attn"
        if config.q_lora_rank is None:
            out[f"{ba}.q_proj.weight"] = hf_sd[f"{a}.q_proj.weight"]
        else:
            out[f"{ba}.q_a_proj.weight"] = hf_sd[f"{a}.q_a_proj.weight"]
            out[f"{ba}.q_a_layernorm.weight"] = hf_sd[f"{a}.q_a_layernorm.weight"]
            out[f"{ba}.q_b_proj.weight"] = hf_sd[f"{a}.q_b_proj.weight"]
        out[f"{ba}.kv_a_proj.weight"] = hf_sd[f"{a}.kv_a_proj_with_mqa.weight"]
        out[f"{ba}.kv_a_layernorm.weight"] = hf_sd[f"{a}.kv_a_layernorm.weight"]
        out[f"{ba}.kv_b_proj.weight"] = hf_sd[f"{a}.kv_b_proj.weight"]
        out[f"{ba}.o_proj.weight"] = hf_sd[f"{a}.o_proj.weight"]
        bf = f"{b}.ffn"
        if i < config.first_k_dense_replace or config.n_routed_experts == 0:
            _fused_mlp(hf_sd, f"{p}.mlp", bf, out)
            continue
        out[f"{bf}.router.gate.weight"] = hf_sd[f"{p}.mlp.gate.weight"]
        out[f"{bf}.router.e_score_correction_bias"] = hf_sd.get(
            f"{p}.mlp.gate.e_score_correction_bias", torch.zeros(config.n_routed_experts)
        )
        for e in range(config.n_routed_experts):
            _fused_mlp(hf_sd, f"{p}.mlp.experts.{e}", f"{bf}.experts.{e}", out)
        if config.n_shared_experts:
            _fused_mlp(hf_sd, f"{p}.mlp.shared_experts", f"{bf}.shared_experts.0", out)
    return out
