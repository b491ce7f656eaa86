"""priml_b200: a Blackwell-native (B200 / sm_100a) training framework.

Public packages mirror the reference's layout: ``config`` (config trees),
``models`` (blocks), ``optimizers``, ``loss``, ``metrics``, ``math``, ``data``,
``train`` (loop, step, checkpointing, strategies), ``parallel`` (runtime,
FSDP / TP / EP engines, symmetric memory), ``ops`` (sm_100a kernels),
``inference``, ``hub`` and ``cost``.
"""

__version__ = "0.1.0"
