"""Test utilities: multi-rank CPU harness (gloo), golden-file helpers."""

from priml_b200.testing.worker_pool import WorkerPool, free_port, run_ranks

__all__ = ["WorkerPool", "free_port", "run_ranks"]
