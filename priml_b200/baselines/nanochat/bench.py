"""Train throughput of the nanochat recipe on synthetic tokens (device-timed).

    python -m priml_b200.baselines.nanochat.bench [--steps 5] [--warmup 2] [--rows-per-pass 64]

The exp000 geometry (d512, 8 layers, S=2048, vocab 8192, SSSL windows, value
embeddings on alternating layers, bf16 tables), 524,288 tokens per optimizer
step by accumulation, the full NorMuon + 5 x AdamW update. Uniform random
tokens (no corpus on the box). Timed with CUDA events around whole optimizer
steps after warm-up; prints one JSON line.
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--rows-per-pass", type=int, default=64)
    args = ap.parse_args()
    from priml_b200.baselines.nanochat.experiments import exp000

    torch.manual_seed(0)
    cfg = exp000()
    step_cfg = cfg.step
    step_cfg.rows_per_pass = args.rows_per_pass
    step_cfg.budget_warmup_steps = 0
    step = step_cfg.make()
    model = step.model
    seq = step_cfg.model.max_seq_len
    vocab = step_cfg.model.vocab_size
    rows = args.rows_per_pass
    g = torch.Generator(device="cuda").manual_seed(1)
    batches = [torch.randint(0, vocab, (rows, seq + 1), device="cuda", generator=g) for _ in range(2)]

    def one_step(i: int) -> None:
        for p in range(step.accumulate_passes):
            b = batches[(i + p) % 2]
            step.train_step(media=b[:, :-1], label=b[:, 1:])

    for i in range(args.warmup):
        one_step(i)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        one_step(i)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    tokens = step_cfg.tokens_per_optimizer_step
    params = sum(p.numel() for p in model.parameters())
    fpt = model.flops_per_token()
    tps = tokens / (ms / 1e3)
    print(json.dumps({"metric": "nanochat train tokens/s (1 GPU, device-timed)", "value": round(tps, 1),
                      "ms_per_step": round(ms, 2), "tokens_per_step": tokens, "rows_per_pass": rows,
                      "params_M": round(params / 1e6, 2), "flops_per_token": fpt,
                      "tflops": round(tps * fpt / 1e12, 1), "last_loss": float(step.last_loss),
                      "data": "synthetic uniform tokens"}))  # fmt: skip


if __name__ == "__main__":
    main()
