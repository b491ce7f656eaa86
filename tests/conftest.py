"""Test configuration: the ``gpu`` marker and CPU-friendly defaults."""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

os.environ.setdefault("OMP_NUM_THREADS", "4")


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")
    config.addinivalue_line("markers", "slow: long-running test")
    for name in ("cuda", "performance", "integration"):  # selector marks that resource markers imply
        config.addinivalue_line("markers", f"{name}: implied by a resource marker")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    has_gpu = torch.cuda.is_available()
    n_gpu = torch.cuda.device_count() if has_gpu else 0
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    skip_multi = pytest.mark.skip(reason="needs >= 2 CUDA devices")
    for item in items:
        if "gpu" in item.keywords and not has_gpu:
            item.add_marker(skip_gpu)
        if "multigpu" in item.keywords and n_gpu < 2:
            item.add_marker(skip_multi)
