from priml_b200.parallel import runtime, strategies  # noqa: F401
