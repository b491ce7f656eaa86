"""Test utilities: multi-rank CPU harness (gloo), bit-for-bit golden files, fixtures."""

from priml_b200.testing.bfb import (
    assert_bfb_against_golden,
    bfb_devices,
    host_agnostic_numerics,
    move_to_device,
    randomize_parameters,
    regenerate_golden,
)
from priml_b200.testing.fixtures import cleanup_cuda, get_device, poison_free_pool, torch_compiler_isolation
from priml_b200.testing.worker_pool import WorkerPool, free_port, run_ranks

__all__ = [
    "WorkerPool",
    "assert_bfb_against_golden",
    "bfb_devices",
    "cleanup_cuda",
    "free_port",
    "get_device",
    "host_agnostic_numerics",
    "move_to_device",
    "poison_free_pool",
    "randomize_parameters",
    "regenerate_golden",
    "run_ranks",
    "torch_compiler_isolation",
]
