"""Alias of :mod:`priml_b200.parallel.runtime` at the reference's import path (``priml.runtime``)."""

from priml_b200.parallel.runtime import *  # noqa: F403
from priml_b200.parallel.runtime import (  # noqa: F401
    MultiProcess,
    SingleProcess,
    destroy_global_device_mesh,
    get_device,
    global_device_mesh,
    initialize_global_device_mesh,
    is_rank_zero,
    runtime_initialized,
)
