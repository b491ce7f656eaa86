"""Model blocks with the reference's public names and parameter layouts
(``priml/model/__init__.py``)."""

from priml_b200.models.attention import (
    MultiStreamAttention,
    OutputGate,
    SdpaFused,
    SdpaNaive,
    SelfAttention,
    layer_window,
    window_mask,
    window_sizes,
)
from priml_b200.models.causal_lm import CausalLM
from priml_b200.models.custom_types import (
    ChannelsIn,
    ChannelsInOut,
    ChannelsOut,
    HasDepth,
    HeadGeometry,
    ShardableConfig,
    ShardStyle,
    propagate_attr,
)
from priml_b200.models.embedding import Embedding, NarrowEmbedding
from priml_b200.models.gated_delta_net import GatedDeltaNet
from priml_b200.models.generate import generate
from priml_b200.models.init import (
    call_init,
    dirac,
    kaiming_normal,
    kaiming_uniform,
    mup_output,
    normal,
    truncated_normal,
    unit_fan_in_uniform,
    xavier_normal,
    xavier_uniform,
)
from priml_b200.models.kvcache import KVCache
from priml_b200.models.linear import EnsembleLinear, Linear
from priml_b200.models.mla import MultiHeadLatentAttention
from priml_b200.models.moe import MoE, Router
from priml_b200.models.norm import (
    BatchNorm,
    BatchNorm2d,
    BatchRenorm,
    CenteredRMSNorm,
    GroupNorm,
    GroupNorm2d,
    LayerNorm,
    RMSNorm,
)
from priml_b200.models.rope import RoPE, RoPEMixed, YarnScaling, rotate_conjugate
from priml_b200.models.special import Identity, ResidualMix, Sequential, Skip, SoftCap
from priml_b200.models.swiglu import SwiGLU, SwiGLUReluSquared
from priml_b200.models.transformer import TransformerBlock
from priml_b200.models.value_gated_attention import ValueGatedAttention
from priml_b200.models.vision import (
    AdaLNZero,
    Conv1d,
    Conv2d,
    Conv3d,
    MLPMixerBlock,
    MMDiTBlock,
    Patchify,
    PCAWhiteningConv2d,
    Unpatchify,
)

from priml_b200.models.init import InitFn
from priml_b200.models.kimi_k2 import KimiK2
from priml_b200.models.norm import NormConfigProtocol, NormProtocol
from priml_b200.models.qwen3 import Qwen3

__all__ = [
    "AdaLNZero",
    "BatchNorm",
    "BatchNorm2d",
    "BatchRenorm",
    "CausalLM",
    "CenteredRMSNorm",
    "ChannelsIn",
    "ChannelsInOut",
    "ChannelsOut",
    "Conv1d",
    "Conv2d",
    "Conv3d",
    "Embedding",
    "EnsembleLinear",
    "GatedDeltaNet",
    "GroupNorm",
    "GroupNorm2d",
    "HasDepth",
    "HeadGeometry",
    "Identity",
    "InitFn",
    "KVCache",
    "KimiK2",
    "LayerNorm",
    "Linear",
    "MLPMixerBlock",
    "MMDiTBlock",
    "MoE",
    "MultiHeadLatentAttention",
    "MultiStreamAttention",
    "NarrowEmbedding",
    "NormConfigProtocol",
    "NormProtocol",
    "OutputGate",
    "PCAWhiteningConv2d",
    "Patchify",
    "Qwen3",
    "RMSNorm",
    "ResidualMix",
    "RoPE",
    "RoPEMixed",
    "Router",
    "SdpaFused",
    "SdpaNaive",
    "SelfAttention",
    "Sequential",
    "ShardStyle",
    "ShardableConfig",
    "Skip",
    "SoftCap",
    "SwiGLU",
    "SwiGLUReluSquared",
    "TransformerBlock",
    "Unpatchify",
    "ValueGatedAttention",
    "YarnScaling",
    "call_init",
    "dirac",
    "generate",
    "kaiming_normal",
    "kaiming_uniform",
    "layer_window",
    "mup_output",
    "normal",
    "propagate_attr",
    "rotate_conjugate",
    "truncated_normal",
    "unit_fan_in_uniform",
    "window_mask",
    "window_sizes",
    "xavier_normal",
    "xavier_uniform",
]
