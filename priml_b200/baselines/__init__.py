"""Reference workloads rebuilt on this framework (``priml/baselines``)."""
