"""GroupIndex (crates/tambear/src/group_index.rs:43-204): the persistent row -> group mapping
of a dense int32 key column, built on the GPU (the reference builds it on the host)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class GroupIndex:
    """Device tensors (int32 holding the reference's u32 values):
    row_to_group[i] = keys[i]; group_counts[g]; group_offsets[g] = rows of groups < g (length
    accumulator_size + 1, the last = n_rows); rows_by_group = row ids by group, row order kept."""
    row_to_group: object
    group_counts: object
    group_offsets: object
    rows_by_group: object
    accumulator_size: int
    n_rows: int
    n_active: int

    @classmethod
    def build(cls, ctx, keys, max_key: int) -> "GroupIndex":
        """GroupIndex::build: keys is an int32 device tensor with values in [0, max_key]."""
        o = ctx.group_index_build(keys, max_key)
        return cls(o["row_to_group"], o["group_counts"], o["group_offsets"], o["rows_by_group"], int(max_key) + 1,
                   int(keys.numel()), o["n_active"])

    def is_valid_for(self, keys) -> bool:
        """The reference's O(1) validity check: same length as the indexed column."""
        return int(keys.numel()) == self.n_rows

    def mask_word_count(self) -> int:
        return (self.accumulator_size + 63) // 64
