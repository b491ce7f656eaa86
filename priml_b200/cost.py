"""Analytical cost model: FLOPs, HBM bytes, NVLink bytes and roofline times.

The reference's only cost model is ``NanoChatLM.flops_per_token``
(``priml/baselines/nanochat/model.py:392-422``: 6 x non-embedding params plus the
attention term). This module generalizes it to the model families here and to
the collective traffic of each parallel layout, against the MEASURED peaks in
``MEASURED_PEAKS.json`` (falling back to 1.59 PFLOP/s bf16, 6.65 TB/s HBM and
770 GB/s per-direction NVLink peer bandwidth).
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

__all__ = [
    "DenseLMShape",
    "MLAMoEShape",
    "Peaks",
    "attention_flops",
    "fsdp_nvlink_bytes_per_step",
    "load_peaks",
    "mfu",
    "roofline_time",
    "train_flops_per_token",
]


@dataclass(frozen=True)
class Peaks:
    bf16_tflops: float = 1590.0
    bf16_tflops_sustained: float = 1400.0
    hbm_gbs: float = 6650.0
    nvlink_gbs: float = 770.0
    source: str = "fallback"


def load_peaks(path: str | Path | None = None) -> Peaks:
    p = Path(path) if path is not None else Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return Peaks(
            bf16_tflops=float(d["bf16_tflops"]),
            bf16_tflops_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
            hbm_gbs=float(d["hbm_gbs"]),
            source="measured",
        )
    except (OSError, KeyError, ValueError):
        return Peaks()


@dataclass(frozen=True)
class DenseLMShape:
    """Llama-style decoder: GQA attention + SwiGLU."""

    d_model: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_hidden: int
    vocab: int
    tied: bool = False

    def params_per_layer(self) -> int:
        d, hd = self.d_model, self.head_dim
        attn = d * (self.n_heads + 2 * self.n_kv_heads) * hd + self.n_heads * hd * d
        mlp = 3 * d * self.ffn_hidden
        return attn + mlp

    def matmul_params(self) -> int:
        """Parameters that take part in a GEMM per token (embedding lookup excluded)."""
        return self.n_layers * self.params_per_layer() + self.vocab * self.d_model

    def total_params(self) -> int:
        emb = self.vocab * self.d_model
        return self.n_layers * self.params_per_layer() + emb * (1 if self.tied else 2)


@dataclass(frozen=True)
class MLAMoEShape:
    d_model: int
    n_layers: int
    n_heads: int
    kv_lora_rank: int
    qk_nope: int
    qk_rope: int
    v_head: int
    dense_hidden: int
    first_dense: int
    n_experts: int
    top_k: int
    expert_hidden: int
    n_shared: int
    vocab: int

    def active_matmul_params(self) -> int:
        d, h = self.d_model, self.n_heads
        attn = (d * h * (self.qk_nope + self.qk_rope) + d * (self.kv_lora_rank + self.qk_rope)
                + self.kv_lora_rank * h * (self.qk_nope + self.v_head) + h * self.v_head * d)  # fmt: skip
        dense = 3 * d * self.dense_hidden
        moe = 3 * d * self.expert_hidden * (self.top_k + self.n_shared) + d * self.n_experts
        layers = self.first_dense * (attn + dense) + (self.n_layers - self.first_dense) * (attn + moe)
        return layers + self.vocab * d


def attention_flops(seq: int, n_heads: int, d_qk: int, d_v: int, causal: bool = True) -> float:
    """Forward attention FLOPs per token per layer: 2*S*(d_qk + d_v)*H, halved when causal."""
    f = 2.0 * seq * (d_qk + d_v) * n_heads
    return f / 2 if causal else f


def train_flops_per_token(shape: DenseLMShape | MLAMoEShape, seq: int) -> float:
    """Model FLOPs per trained token: 6 x GEMM params + 3 x forward attention (fwd + 2x bwd)."""
    if isinstance(shape, DenseLMShape):
        attn = attention_flops(seq, shape.n_heads, shape.head_dim, shape.head_dim) * shape.n_layers
        return 6.0 * shape.matmul_params() + 3.0 * attn
    attn = attention_flops(seq, shape.n_heads, shape.qk_nope + shape.qk_rope, shape.v_head) * shape.n_layers
    return 6.0 * shape.active_matmul_params() + 3.0 * attn


def mfu(tokens_per_s: float, flops_per_token: float, n_gpus: int = 1, peaks: Peaks | None = None,
        sustained: bool = True) -> float:  # fmt: skip
    p = peaks or load_peaks()
    peak = p.bf16_tflops_sustained if sustained else p.bf16_tflops
    return tokens_per_s * flops_per_token / (n_gpus * peak * 1e12)


def fsdp_nvlink_bytes_per_step(n_params: int, world: int, *, param_bytes: int = 2, grad_bytes: int = 4,
                               regather_in_backward: bool = True) -> float:  # fmt: skip
    """Bytes each GPU sends over NVLink per step under FSDP (ring-equivalent):
    all-gather of params (once, twice with re-gather in backward) plus the
    gradient reduce-scatter, each moving ``(world-1)/world`` of the full tensor."""
    if world <= 1:
        return 0.0
    frac = (world - 1) / world
    ag = n_params * param_bytes * frac * (2 if regather_in_backward else 1)
    rs = n_params * grad_bytes * frac
    return ag + rs


def roofline_time(flops: float, nvlink_bytes: float = 0.0, hbm_bytes: float = 0.0, peaks: Peaks | None = None) -> float:
    """Seconds at the slower of compute, HBM and NVLink rooflines."""
    p = peaks or load_peaks()
    return max(flops / (p.bf16_tflops * 1e12), hbm_bytes / (p.hbm_gbs * 1e9), nvlink_bytes / (p.nvlink_gbs * 1e9))


LLAMA_1B = DenseLMShape(d_model=2048, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64, ffn_hidden=8192, vocab=32768)
LLAMA3_8B = DenseLMShape(d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn_hidden=14336, vocab=128256)
MLA_MOE_CFG3 = MLAMoEShape(d_model=2048, n_layers=27, n_heads=16, kv_lora_rank=512, qk_nope=128, qk_rope=64, v_head=128,
                           dense_hidden=10944, first_dense=1, n_experts=64, top_k=6, expert_hidden=1408, n_shared=2,
                           vocab=102400)  # fmt: skip
