"""Support library: JSON helpers, object traversal, XDG user dirs (``priml/lib``)."""

from priml_b200.lib.misc import (
    bool_val,
    dict_val,
    float_val,
    int_val,
    json_freeze,
    json_unfreeze,
    traverse,
    user_cache_dir,
    user_data_dir,
    validate_json_schema,
)

__all__ = [
    "bool_val",
    "dict_val",
    "float_val",
    "int_val",
    "json_freeze",
    "json_unfreeze",
    "traverse",
    "user_cache_dir",
    "user_data_dir",
    "validate_json_schema",
]
