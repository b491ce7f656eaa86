"""Inference: autoregressive decoding for serving.

The reference ships ``priml/inference/__init__.py`` empty and decodes through
``priml/model/generate.py``; that loop is :func:`priml_b200.models.generate.generate`
here. This package adds the serving side:

* :class:`StaticKVCache` / :class:`CacheState` -- fixed KV buffers whose fill
  levels live on the device, with a decode-attention kernel that reads them there;
* :class:`Decoder` -- prefill per row range, then one CUDA graph replay per token
  for the whole batch;
* :func:`sample` / :class:`SamplingParams` -- per-row temperature / top-k / top-p
  drawn on the device (Gumbel-max), capturable in the same graph.
"""

from priml_b200.inference.cache import CacheState, StaticKVCache
from priml_b200.inference.decoder import Decoder
from priml_b200.inference.sampling import SamplingParams, sample
from priml_b200.models.generate import generate, sample_logits

__all__ = ["CacheState", "Decoder", "SamplingParams", "StaticKVCache", "generate", "sample", "sample_logits"]
