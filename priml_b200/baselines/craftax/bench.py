"""Craftax PPO training throughput in environment steps per second (device-timed).

    python -m priml_b200.baselines.craftax.bench [--envs 1024] [--rollout 64] [--steps 3] [--warmup 1]

The exp001 geometry: 1,024 workers, 64-step rollouts, PPO update on the
8,268-float observation (the reference quotes its Craftax PPO throughput in
environment steps per second, ``priml/train/tracker.py:476-481``). Every timed
update collects ``envs x rollout`` steps of the batched game on the device and
trains on them; steps/s = envs x rollout x updates / CUDA-event time. Prints
one JSON line.
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--envs", type=int, default=1024)
    ap.add_argument("--rollout", type=int, default=64)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--device", default="cuda")
    args = ap.parse_args()
    from priml_b200.baselines.craftax import CraftaxEnv, CraftaxTrainStep

    cfg = CraftaxTrainStep.Config()
    cfg.env = CraftaxEnv.Config(num_envs=args.envs, device=args.device, seed=0)
    cfg.rollout_steps = args.rollout
    cfg.learning_rate = 2e-4
    step = cfg.make()
    cuda = torch.device(args.device).type == "cuda"
    for _ in range(args.warmup):
        step.train_step()
    if cuda:
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    else:
        import time

        t0 = time.perf_counter()
    for _ in range(args.steps):
        out = step.train_step()
    if cuda:
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / args.steps
    else:
        ms = (time.perf_counter() - t0) * 1e3 / args.steps
    env_steps = args.envs * args.rollout
    print(json.dumps({"metric": "Craftax PPO env steps/s (1 GPU, device-timed)" if cuda else "Craftax PPO env steps/s (CPU)",
                      "value": round(env_steps / (ms / 1e3), 1), "unit": "steps/s", "ms_per_update": round(ms, 2),
                      "config": {"envs": args.envs, "rollout": args.rollout, "updates": args.steps, "warmup": args.warmup},
                      "loss": float(out["loss"])}))  # fmt: skip


if __name__ == "__main__":
    main()
