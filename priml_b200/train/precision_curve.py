"""Loss curves of the same run in bf16 and with MXFP8 linear layers.

    python -m priml_b200.train.precision_curve [--layers 2] [--steps 200] [--out curve.txt]

Model: the Llama-3-8B layer shape (d 4096, 32 / 8 heads x 128, SwiGLU 14336, vocab
128256) at the given depth. Data: a synthetic language with learnable structure over the
first 512 token ids -- every token has four successors fixed by a hash of the token,
one drawn uniformly at each step -- so the loss falls from log(vocab) through
log(512) toward log(4) = 1.386 nats, and a precision problem shows up as a gap
between the curves. Both runs start from the same
weights and see the same batches; the optimizer is FusedAdamW with clipping. The
output lists both curves step by step and their largest and final gaps.
"""

from __future__ import annotations

import argparse
import json
import math
import time
from pathlib import Path

import torch

__all__ = ["markov_batch", "run_curve"]


def markov_batch(batch: int, seq: int, vocab: int, generator: torch.Generator, device: torch.device) -> torch.Tensor:
    """``[batch, seq + 1]`` tokens of the four-successor language."""
    tok = torch.randint(0, vocab, (batch,), generator=generator, device=device)
    out = [tok]
    mult = torch.tensor([1_000_003, 999_983, 1_000_033, 999_979], device=device)
    for _ in range(seq):
        pick = torch.randint(0, 4, (batch,), generator=generator, device=device)
        tok = (tok * mult[pick] + 7919 * (pick + 1)) % vocab
        out.append(tok)
    return torch.stack(out, dim=1)


def run_curve(*, layers: int, steps: int, mxfp8: bool, seq: int = 2048, batch: int = 2, d_model: int = 4096,
              heads: int = 32, kv_heads: int = 8, head_dim: int = 128, ffn: int = 14336, vocab: int = 128256,
              lr: float = 3e-4, seed: int = 0) -> list[float]:  # fmt: skip
    from priml_b200.loss import TokenCrossEntropy
    from priml_b200.models.presets import dense_lm
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.parallel.strategies import NoParallel
    from priml_b200.train import Float8ModelQuantization, TrainStep

    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(seed)
    kw = {"model_quantization": Float8ModelQuantization.Config(recipe="mxfp8")} if mxfp8 else {}
    step = TrainStep.Config(
        model=dense_lm(vocab=vocab, d_model=d_model, n_layers=layers, n_heads=heads, n_kv_heads=kv_heads,
                       head_dim=head_dim, ffn_hidden=ffn, rope_theta=5e5),  # fmt: skip
        optimizer=FusedAdamW.Config(lr=lr, betas=(0.9, 0.95), weight_decay=0.1),
        loss=TokenCrossEntropy.Config(),
        parallelism=NoParallel.Config(),
        dtype_autocast=torch.bfloat16,
        gradient_clip_norm=1.0,
        **kw,
    ).make()
    step.model.to(dev)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    losses = []
    for _ in range(steps):
        seqs = markov_batch(batch, seq, min(vocab, 512), g, dev)
        out = step.train_step(tokens=seqs[:, :-1], targets=seqs[:, 1:])
        losses.append(float(out["loss"].detach().float().mean()))
    return losses


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--out", type=str, default="")
    args = ap.parse_args()
    t0 = time.time()
    bf16 = run_curve(layers=args.layers, steps=args.steps, mxfp8=False, seq=args.seq, batch=args.batch)
    mx = run_curve(layers=args.layers, steps=args.steps, mxfp8=True, seq=args.seq, batch=args.batch)
    gaps = [abs(a - b) for a, b in zip(bf16, mx, strict=True)]
    tail = max(1, len(gaps) // 4)
    summary = {
        "model": f"llama-3-8b layer shape, {args.layers} layers, vocab 128256", "steps": args.steps,
        "tokens_per_step": args.seq * args.batch, "floor_nats": math.log(4),
        "bf16_first_last": [round(bf16[0], 4), round(bf16[-1], 4)], "mxfp8_first_last": [round(mx[0], 4), round(mx[-1], 4)],
        "max_abs_gap": round(max(gaps), 4), "mean_abs_gap_last_quarter": round(sum(gaps[-tail:]) / tail, 4),
        "wall_s": round(time.time() - t0, 1),
    }  # fmt: skip
    print(json.dumps(summary), flush=True)
    if args.out:
        lines = ["step\tbf16\tmxfp8"] + [f"{i}\t{a:.5f}\t{b:.5f}" for i, (a, b) in enumerate(zip(bf16, mx, strict=True))]
        Path(args.out).write_text(json.dumps(summary) + "\n" + "\n".join(lines) + "\n")


if __name__ == "__main__":
    main()
