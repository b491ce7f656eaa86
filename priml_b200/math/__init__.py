from priml_b200.math import basic, distributed, loss, numeric, schedules, seed  # noqa: F401
