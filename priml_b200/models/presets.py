"""Model presets for the benchmark workloads.

* ``tiny_lm``      vocab 512, d 128, 2 layers, 4 heads x 32, SwiGLU 512, RoPE 1e4 (fp32 CPU check).
* ``tiny_moe_lm``  tiny_lm with MoE FFNs: 8 routed SwiGLU experts x 128 (top-2 softmax) + 1 shared.
* ``llama_1b``     d 2048, 16 layers, 32 q / 8 kv heads x 64, SwiGLU 8192, RMSNorm 1e-5,
                   RoPE 5e5, vocab 32768, untied, init N(0, 0.02).
* ``llama3_8b``    d 4096, 32 layers, 32 / 8 heads x 128, SwiGLU 14336, RoPE 5e5, vocab 128256.
* ``mla_moe``      MLA (16 heads, kv_lora 512, nope 128, rope 64, v 128) + MoE (64 routed
                   experts x 1408, top-6 softmax, 2 shared; first layer dense 10944), vocab 102400.
"""

from __future__ import annotations

from functools import partial

from priml_b200.config import copy_tree
from priml_b200.models.attention import SelfAttention
from priml_b200.models.causal_lm import CausalLM
from priml_b200.models.embedding import Embedding
from priml_b200.models.init import normal
from priml_b200.models.linear import Linear
from priml_b200.models.mla import MultiHeadLatentAttention
from priml_b200.models.moe import MoE, Router
from priml_b200.models.norm import RMSNorm
from priml_b200.models.rope import RoPE
from priml_b200.models.swiglu import SwiGLU
from priml_b200.models.transformer import TransformerBlock

__all__ = ["dense_lm", "llama3_8b", "llama_1b", "mla_moe", "tiny_lm", "tiny_moe_lm"]


def dense_lm(
    *,
    vocab: int,
    d_model: int,
    n_layers: int,
    n_heads: int,
    n_kv_heads: int,
    head_dim: int,
    ffn_hidden: int,
    rope_theta: float,
    norm_eps: float = 1e-5,
    init_std: float | None = 0.02,
    checkpoint: bool = False,
) -> CausalLM.Config:
    init = partial(normal, std=init_std) if init_std is not None else None
    attn_kw = {"init_weight": init} if init is not None else {}
    ffn_kw = {"init_weight": init} if init is not None else {}
    block = TransformerBlock.Config(
        attn=SelfAttention.Config(
            heads=n_heads,
            channels_head=head_dim,
            num_heads_kv=n_kv_heads,
            causal=True,
            rope=RoPE.Config(head_dim, base=rope_theta),
            **attn_kw,
        ),
        ffn=SwiGLU.Config(channels_hidden=ffn_hidden, **ffn_kw),
        norm1=RMSNorm.Config(eps=norm_eps),
        norm2=RMSNorm.Config(eps=norm_eps),
        checkpoint=checkpoint,
    )
    head = Linear.Config(bias=False, shard="vocab", init_weight=init) if init is not None else None
    embed = Embedding.Config(shard="vocab", init_weight=init) if init is not None else None
    return CausalLM.Config(
        vocab,
        channels=d_model,
        num_layers=n_layers,
        block=block,
        final_norm=RMSNorm.Config(eps=norm_eps),
        lm_head=head,
        embed=embed,
    )


def tiny_lm() -> CausalLM.Config:
    return dense_lm(vocab=512, d_model=128, n_layers=2, n_heads=4, n_kv_heads=4, head_dim=32, ffn_hidden=512,
                    rope_theta=1e4, norm_eps=1e-6, init_std=None)  # fmt: skip


def tiny_moe_lm(*, num_experts: int = 8, top_k: int = 2, aux_loss_weight: float = 0.0) -> CausalLM.Config:
    block = TransformerBlock.Config(
        attn=SelfAttention.Config(heads=4, channels_head=32, causal=True, rope=RoPE.Config(32, base=1e4)),
        ffn=MoE.Config(
            router=Router.Config(num_experts=num_experts, top_k=top_k, scoring_func="softmax"),
            expert=SwiGLU.Config(channels_hidden=128),
            num_shared_experts=1,
            shared_expert=SwiGLU.Config(channels_hidden=128),
            aux_loss_weight=aux_loss_weight,
        ),
        norm1=RMSNorm.Config(eps=1e-6),
        norm2=RMSNorm.Config(eps=1e-6),
    )
    return CausalLM.Config(512, channels=128, num_layers=2, block=block, final_norm=RMSNorm.Config(eps=1e-6))


def llama_1b(*, checkpoint: bool = False) -> CausalLM.Config:
    return dense_lm(vocab=32768, d_model=2048, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64, ffn_hidden=8192,
                    rope_theta=5e5, checkpoint=checkpoint)  # fmt: skip


def llama3_8b(*, checkpoint: bool = True) -> CausalLM.Config:
    return dense_lm(vocab=128256, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128,
                    ffn_hidden=14336, rope_theta=5e5, checkpoint=checkpoint)  # fmt: skip


def mla_moe(*, n_layers: int = 27) -> CausalLM.Config:
    init = partial(normal, std=0.02)
    attn = MultiHeadLatentAttention.Config(
        heads=16,
        kv_lora_rank=512,
        channels_qk_nope_head=128,
        channels_qk_rope_head=64,
        channels_v_head=128,
        rope=RoPE.Config(64, base=1e4),
        init_weight=init,
    )
    dense = TransformerBlock.Config(attn=copy_tree(attn), ffn=SwiGLU.Config(channels_hidden=10944, init_weight=init))
    moe = TransformerBlock.Config(
        attn=copy_tree(attn),
        ffn=MoE.Config(
            router=Router.Config(num_experts=64, top_k=6, scoring_func="softmax"),
            expert=SwiGLU.Config(channels_hidden=1408, init_weight=init),
            num_shared_experts=2,
            shared_expert=SwiGLU.Config(channels_hidden=1408, init_weight=init),
        ),
    )
    # one config tree per layer: finalization writes widths into each block's (and its attention's) config
    return CausalLM.Config(
        102400,
        channels=2048,
        num_layers=n_layers,
        block=[dense] + [copy_tree(moe) for _ in range(n_layers - 1)],
        lm_head=Linear.Config(bias=False, shard="vocab", init_weight=init),
        embed=Embedding.Config(shard="vocab", init_weight=init),
    )
