"""Math library (``priml/math``)."""

from priml_b200.math import (  # noqa: F401
    activations,
    advantage,
    basic,
    custom_types,
    diffusion,
    distributed,
    frequency,
    loss,
    numeric,
    pixel,
    pooling,
    probability,
    schedules,
    seed,
    stats,
    tensor,
)
