"""Batched decoding with static KV caches and one CUDA graph per decode step.

The reference decodes through ``priml/model/generate.py:40-130``: a Python loop
over the blocks for every token, with cache bookkeeping on the host. On a B200 a
small model's decode step is then bound by kernel launches and host work, not by
HBM. :class:`Decoder` keeps every piece of per-step state on the device
(:mod:`priml_b200.inference.cache`), so after the first step the whole token
step -- embedding, every block, the final norm, the logits and the draw -- is
one graph replay:

* ``prefill(tokens, rows)`` runs a prompt for a range of sequences eagerly (flash
  attention over the prompt when those rows are empty) and returns the last
  position's logits;
* ``step(tokens)`` appends one token to every sequence and returns the next token
  of each (sampled in the graph with per-row settings) and the logits;
* ``generate(prompt, ...)`` is the reference's ``generate`` on top of these.

Rows are independent: ``reset(rows)`` empties some sequences and ``prefill`` can
refill them while the others keep their caches, which is what a server that
admits requests into a running batch needs. Every row advances on ``step``;
a finished row simply keeps producing tokens that the caller ignores until it
is reset. The host mirrors each row's length to refuse overflowing the cache
without reading the device.

Models: decoder-only stacks whose blocks use :class:`~priml_b200.models.attention.SelfAttention`
(Llama / Qwen3 dense presets). Multi-head latent attention keeps its latent cache
in :func:`priml_b200.models.generate.generate`.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor, nn

from priml_b200.inference.cache import CacheState, StaticKVCache
from priml_b200.inference.sampling import SamplingParams, sample

__all__ = ["Decoder"]


def _param_dtype(model: nn.Module) -> torch.dtype:
    for p in model.parameters():
        if p.is_floating_point():
            return p.dtype
    return torch.float32


class Decoder:
    """Static-cache decoding for a batch of ``batch`` sequences of up to ``max_seq`` tokens."""

    def __init__(
        self,
        model: nn.Module,
        *,
        batch: int,
        max_seq: int,
        dtype: torch.dtype | None = None,
        cuda_graph: bool = True,
    ) -> None:
        from priml_b200.models.attention import SelfAttention

        blocks = list(getattr(model, "blocks", []))
        if not blocks or not all(isinstance(getattr(b, "attn", None), SelfAttention) for b in blocks):
            raise TypeError("Decoder needs a decoder-only model whose blocks all use SelfAttention.")
        self.model = model.eval()
        self.device = next(model.parameters()).device
        self.dtype = dtype or _param_dtype(model)
        self.batch, self.max_seq = batch, max_seq
        self.state = CacheState.create(batch, max_seq, self.device)
        self.caches = [
            StaticKVCache.alloc(self.state, heads=b.attn.num_heads_kv, channels_head=b.attn.channels_head,
                                device=self.device, dtype=self.dtype)  # fmt: skip
            for b in blocks
        ]
        self.host_lengths = [0] * batch
        self.use_graph = cuda_graph and self.device.type == "cuda"
        self._tok = torch.zeros(batch, dtype=torch.long, device=self.device)
        self._temperature = torch.ones(batch, dtype=torch.float32, device=self.device)
        self._top_k = torch.zeros(batch, dtype=torch.long, device=self.device)
        self._top_p = torch.ones(batch, dtype=torch.float32, device=self.device)
        self._graphs: dict[bool, tuple[torch.cuda.CUDAGraph, Tensor, Tensor]] = {}

    # ------------------------------------------------------------------ state
    def reset(self, rows: slice | None = None) -> None:
        """Empty the caches of ``rows`` (all rows by default)."""
        rows = rows or slice(0, self.batch)
        self.state.lengths[rows] = 0
        for i in range(*rows.indices(self.batch)):
            self.host_lengths[i] = 0

    def set_sampling(self, params: SamplingParams | list[SamplingParams]) -> None:
        """Per-row sampling settings used by :meth:`step` (one value for all rows, or one per row)."""
        plist = params if isinstance(params, list) else [params] * self.batch
        if len(plist) != self.batch:
            raise ValueError(f"need {self.batch} sampling settings, got {len(plist)}.")
        t, k, p = SamplingParams.stack(plist, self.device)
        self._temperature.copy_(t)
        self._top_k.copy_(k)
        self._top_p.copy_(p)
        self._filtered = any(q.filtered for q in plist)

    _filtered = False

    # ------------------------------------------------------------------ forward
    def _forward(self, tokens: Tensor, state: CacheState, caches: list[StaticKVCache]) -> Tensor:
        model: Any = self.model
        s = tokens.shape[1]
        x = model.embed(tokens)
        pos = state.positions(s)
        for block, cache in zip(model.blocks, caches, strict=True):
            x, _ = block(x, cache=cache, positions=pos)
        logits = model.project_to_logits(model.final_norm(x[:, -1]))
        state.advance(s)
        state.lengths.clamp_(max=state.capacity)
        return logits

    @torch.inference_mode()
    def prefill(self, tokens: Tensor, rows: slice | None = None) -> Tensor:
        """Append ``[n, S]`` prompt tokens to ``rows`` (``n`` rows; all by default); returns ``[n, V]`` logits."""
        rows = rows or slice(0, self.batch)
        idx = range(*rows.indices(self.batch))
        if len(idx) != tokens.shape[0] or rows.step not in (None, 1):
            raise ValueError(f"{tokens.shape[0]} prompts for rows {rows}.")
        s = tokens.shape[1]
        if any(self.host_lengths[i] + s > self.max_seq for i in idx):
            raise ValueError(f"a prompt of {s} tokens overflows the {self.max_seq}-token cache.")
        state = self.state.select(rows)
        state.fresh = all(self.host_lengths[i] == 0 for i in idx)
        caches = [c.select(rows, state) for c in self.caches]
        logits = self._forward(tokens.to(self.device), state, caches)
        for i in idx:
            self.host_lengths[i] += s
        return logits

    def _step_body(self, filtered: bool) -> tuple[Tensor, Tensor]:
        logits = self._forward(self._tok[:, None], self.state, self.caches)
        nxt = sample(logits, self._temperature, self._top_k, self._top_p, filtered=filtered)
        return nxt, logits

    def _capture(self, filtered: bool) -> tuple[torch.cuda.CUDAGraph, Tensor, Tensor]:
        saved = self.state.lengths.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._step_body(filtered)  # warm-up: first-use allocations and kernel selection
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.state.lengths.copy_(saved)  # the warm-up's cache rows are rewritten by the real step
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            nxt, logits = self._step_body(filtered)
        return graph, nxt, logits

    @torch.inference_mode()
    def step(self, tokens: Tensor) -> tuple[Tensor, Tensor]:
        """Append one token ``[B]`` to every row; returns ``(next tokens [B], logits [B, V])``.

        The returned tensors are the graph's output buffers: the next call overwrites them.
        """
        if any(0 < n and n + 1 > self.max_seq for n in self.host_lengths):
            raise ValueError(f"a sequence would overflow the {self.max_seq}-token cache.")
        self._tok.copy_(tokens.reshape(-1))
        if self.use_graph:
            entry = self._graphs.get(self._filtered)
            if entry is None:
                entry = self._graphs[self._filtered] = self._capture(self._filtered)
            entry[0].replay()
            nxt, logits = entry[1], entry[2]
        else:
            nxt, logits = self._step_body(self._filtered)
        self.host_lengths = [min(n + 1, self.max_seq) for n in self.host_lengths]
        return nxt, logits

    # ------------------------------------------------------------------ convenience
    @torch.inference_mode()
    def generate(
        self,
        prompt_ids: Tensor,
        *,
        max_new_tokens: int = 128,
        temperature: float = 1.0,
        top_k: int = 0,
        top_p: float = 1.0,
        eos_token_id: int | None = None,
    ) -> Tensor:
        """``[B, S]`` prompt -> ``[B, S + generated]`` tokens; stops early once every row has emitted EOS."""
        if prompt_ids.shape[0] != self.batch:
            raise ValueError(f"the decoder holds {self.batch} rows, the prompt has {prompt_ids.shape[0]}.")
        if prompt_ids.shape[1] + max_new_tokens > self.max_seq:
            raise ValueError(f"prompt + {max_new_tokens} new tokens exceed max_seq={self.max_seq}.")
        self.reset()
        self.set_sampling(SamplingParams(temperature, top_k, top_p))
        logits = self.prefill(prompt_ids)
        tok = sample(logits, self._temperature, self._top_k, self._top_p, filtered=self._filtered)
        out = [tok.clone()]
        done = torch.zeros(self.batch, dtype=torch.bool, device=self.device)
        for _ in range(max_new_tokens - 1):
            if eos_token_id is not None:
                done |= out[-1] == eos_token_id
                if bool(done.all()):
                    break
            tok, _ = self.step(out[-1])
            out.append(tok.clone())
        if max_new_tokens <= 0:
            return prompt_ids
        return torch.cat([prompt_ids.to(self.device), torch.stack(out, dim=-1)], dim=-1)
