"""Shard-spec strings -> shard id sets (``priml/sharding.py:6-74``).

``"1,4:9,::2,-5:"``: comma-separated ids and Python slices over
``range(total_shards)`` (negative indices and steps follow slice semantics).
"""

from __future__ import annotations

__all__ = ["parse_shard_spec"]


def parse_shard_spec(spec: str, total_shards: int) -> set[int]:
    ids: set[int] = set()
    for part in spec.split(","):
        part = part.strip()
        if not part:
            continue
        if ":" in part:
            fields = [f.strip() for f in part.split(":")]
            if len(fields) > 3:
                raise ValueError(f"bad slice {part!r}")
            start, stop, step = (int(f) if f else None for f in (fields + ["", ""])[:3])
            ids.update(range(*slice(start, stop, step).indices(total_shards)))
        else:
            i = int(part)
            if i < 0:
                i += total_shards
            if not 0 <= i < total_shards:
                raise ValueError(f"shard {part} out of range for {total_shards} shards")
            ids.add(i)
    return ids
