"""Hugging Face checkpoint access (``priml/hub.py:31-221``).

Local directory first; otherwise ``huggingface_hub.snapshot_download`` (cache
first) when that package is importable. Weights load from ``*.safetensors`` or
``pytorch_model*.bin`` shards into one flat state dict.
"""

from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Any

import torch

__all__ = ["load_config", "load_local_state_dict", "load_transformers_model", "resolve_hf_dtype", "resolve_local_path"]

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "fp32": torch.float32,
           "fp16": torch.float16, "bf16": torch.bfloat16}  # fmt: skip


def resolve_hf_dtype(config: dict[str, Any], override: torch.dtype | None = None) -> torch.dtype:
    if override is not None:
        return override
    name = config.get("torch_dtype") or config.get("dtype") or "float32"
    return _DTYPES.get(str(name).replace("torch.", ""), torch.float32)


def resolve_local_path(path_or_repo: str | Path) -> Path:
    p = Path(path_or_repo)
    if p.is_dir():
        return p
    try:
        from huggingface_hub import snapshot_download  # type: ignore[import-not-found]
    except ImportError as exc:  # pragma: no cover - depends on the image
        raise FileNotFoundError(f"{path_or_repo} is not a local directory and huggingface_hub is unavailable") from exc
    cache = os.environ.get("TORCH_HOME")
    return Path(snapshot_download(str(path_or_repo), cache_dir=cache))


def load_config(path: str | Path) -> dict[str, Any]:
    return json.loads((resolve_local_path(path) / "config.json").read_text())


def load_local_state_dict(path: str | Path, *, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    root = resolve_local_path(path)
    out: dict[str, torch.Tensor] = {}
    st = sorted(root.glob("*.safetensors"))
    if st:
        from safetensors.torch import load_file

        for f in st:
            out.update(load_file(str(f), device=str(device)))
        return out
    bins = sorted(root.glob("pytorch_model*.bin"))
    if not bins:
        raise FileNotFoundError(f"no *.safetensors or pytorch_model*.bin under {root}")
    for f in bins:
        out.update(torch.load(f, map_location=device, weights_only=True))
    return out


def load_transformers_model(path_or_repo: str | Path, **kwargs: Any) -> Any:
    """The HF ``AutoModelForCausalLM`` for parity tests (eager attention)."""
    from transformers import AutoModelForCausalLM

    kwargs.setdefault("attn_implementation", "eager")
    return AutoModelForCausalLM.from_pretrained(str(resolve_local_path(path_or_repo)), **kwargs)
