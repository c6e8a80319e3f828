"""Host-side logic of the Python caller surface (no GPU): FilterJit predicate parsing and the
header-only tile-statistics queries (format.rs:144-175) on a host TileColumnStats array."""
import math

import numpy as np
import pytest

from winrapids_b200 import EntryNotFound
from winrapids_b200.frame import (PRED_FINITE, PRED_GT, PRED_NOT_NAN, PRED_POSITIVE, TILE_STATS_DTYPE,
                                  parse_predicate)


@pytest.mark.parametrize("expr,want", [
    (PRED_GT + "110.0", (">", 110.0)), ("v > 4.0", (">", 4.0)), ("v>=-2.5", (">=", -2.5)),
    ("  v <  1e3 ", ("<", 1000.0)), ("v <= .5", ("<=", 0.5)), (PRED_POSITIVE, (">", 0.0)),
    ("v > inf", (">", math.inf)), (PRED_NOT_NAN, ("not_nan", 0.0)), (PRED_FINITE, ("finite", 0.0)),
    ("v  ==  v", ("not_nan", 0.0)),
])
def test_parse_predicate(expr, want):
    got = parse_predicate(expr)
    assert got[0] == want[0] and got[1] == want[1]


def test_parse_predicate_nan_threshold():
    p, t = parse_predicate("v > nan")
    assert p == ">" and math.isnan(t)


@pytest.mark.parametrize("expr", ["v * 2 > 1", "x > 1", "v > ", "v != 3", "v > 1 && v < 2", ""])
def test_parse_predicate_rejects(expr):
    with pytest.raises(EntryNotFound):
        parse_predicate(expr)


def test_tile_stats_dtype_is_the_40_byte_layout():
    assert TILE_STATS_DTYPE.itemsize == 40
    assert [TILE_STATS_DTYPE.fields[f][1] for f in ("min", "max", "sum", "count", "n_valid", "reserved")] == \
        [0, 8, 16, 24, 28, 32]


def test_global_queries_on_host_stats(monkeypatch):
    """global_min / _max / _sum / _count / _mean (format.rs:144-175) over stats, with a NaN tile
    min that Rust's f64::min skips and an empty tile that the n_valid filter skips."""
    from winrapids_b200 import frame

    st = np.zeros(3, TILE_STATS_DTYPE)
    st[0] = (1.0, 5.0, 9.0, 3, 3, 0)
    st[1] = (math.nan, 7.0, 12.0, 2, 2, 0)
    st[2] = (-100.0, 100.0, 0.0, 0, 0, 0)  # n_valid 0: ignored by min / max
    monkeypatch.setattr(frame, "tile_stats_numpy", lambda s: s)
    assert frame.global_min(st) == 1.0 and frame.global_max(st) == 7.0
    assert frame.global_sum(st) == 21.0 and frame.global_count(st) == 5
    assert frame.global_mean(st) == 21.0 / 5
    empty = np.zeros(0, TILE_STATS_DTYPE)
    assert math.isnan(frame.global_mean(empty)) and frame.global_min(empty) == math.inf
