"""Diffusion math: schedules, prediction targets, samplers (``priml/math/diffusion``)."""

from priml_b200.math.diffusion.sampling import *  # noqa: F403
from priml_b200.math.diffusion.schedule import *  # noqa: F403
from priml_b200.math.diffusion.target import *  # noqa: F403
