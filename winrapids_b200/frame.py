"""Mask-not-filter plumbing and the Python caller surface, over the C ABI.

Mirrors, with the reference's names and meaning:

* ``FilterJit.filter_mask`` (crates/tambear/src/filter_jit.rs:71-121): a predicate string
  over ``v`` -> packed u64 row mask.  The reference JIT-compiles any C expression; the
  predicates accepted here are the ones it names (``PRED_GT`` "v > t", ``PRED_NOT_NAN``
  "v == v", ``PRED_FINITE`` "v == v && v * 0.0 == 0.0", ``PRED_POSITIVE`` "v > 0.0",
  :252-263) and the other comparisons ``v >= t``, ``v < t``, ``v <= t``.
* ``MaskOp`` (filter_jit.rs:262-440): AND / OR / XOR / NOT / popcount of device masks,
  with host-array wrappers.
* ``TileColumnStats`` and the header-only queries of the ``.tb`` format
  (crates/tambear/src/format.rs:60-189): per-tile statistics built on the device,
  ``tile_skip_mask_gt`` / ``_lt``, ``global_min`` / ``_max`` / ``_sum`` / ``_count`` / ``_mean``.
* ``Frame`` / ``GroupByBuilder`` / ``GroupByResult`` / ``from_columns``
  (crates/tambear-py/src/lib.rs:72-345) and the core ``Frame``'s mask-not-filter row mask
  (crates/tambear/src/frame.rs:86-160): ``filter`` sets row-mask bits instead of
  compacting, and every aggregation honours the mask.  Columns live on the device.

Every computation runs in the CUDA library; there is no host fallback.
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass, field

import numpy as np

from . import Context, EntryNotFound, InvalidArgument, _torch
from ._lib import TILE_STATS_FIELDS
from .engines import GroupByResult as _OneScanResult

TB_TILE_SIZE_DEFAULT = 65_536  # format.rs:40

# Predicate constants of filter_jit.rs:252-263
PRED_GT = "v > "
PRED_NOT_NAN = "v == v"
PRED_FINITE = "v == v && v * 0.0 == 0.0"
PRED_POSITIVE = "v > 0.0"

TILE_STATS_DTYPE = np.dtype([(n, "<" + t) for n, t in TILE_STATS_FIELDS])

_CMP = re.compile(r"^\s*v\s*(>=|<=|>|<)\s*([-+]?(?:\d+\.?\d*|\.\d+)(?:[eE][-+]?\d+)?|[-+]?inf|nan)\s*$")


def parse_predicate(expr: str) -> tuple[str, float]:
    """(tbgb predicate, threshold) of a FilterJit predicate string."""
    e = " ".join(expr.split())
    if e == PRED_NOT_NAN:
        return "not_nan", 0.0
    if e == PRED_FINITE:
        return "finite", 0.0
    m = _CMP.match(expr)
    if not m:
        raise EntryNotFound(6, f"unsupported predicate {expr!r} (v OP number, {PRED_NOT_NAN!r}, {PRED_FINITE!r})")
    return m.group(1), float(m.group(2))


_CTX: dict[int, Context] = {}


def _ctx(device: int) -> Context:
    if device not in _CTX:
        _CTX[device] = Context(device)
    return _CTX[device]


def _dev(device: int) -> str:
    return f"cuda:{device}"


def _to_device_words(mask, device: int):
    torch = _torch()
    if isinstance(mask, torch.Tensor):
        return mask.to(_dev(device))
    w = np.ascontiguousarray(np.asarray(mask, dtype=np.uint64)).view(np.int64)
    return torch.from_numpy(w.copy()).to(_dev(device))


def _to_host_words(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint64).copy()


class FilterJit:
    """FilterJit (filter_jit.rs:40-121): predicate -> packed row mask."""

    def __init__(self, device: int = 0):
        self.device = device
        self.ctx = _ctx(device)
        self.cache: dict[str, tuple[str, float]] = {}  # parsed predicates, like the reference's kernel cache

    def _pred(self, expr: str) -> tuple[str, float]:
        if expr not in self.cache:
            self.cache[expr] = parse_predicate(expr)
        return self.cache[expr]

    def filter_mask_gpu(self, expr: str, values, in_mask=None):
        """Device column in, device mask out (int64 words holding the u64 bits)."""
        pred, thr = self._pred(expr)
        return self.ctx.filter_mask(values, pred, thr, in_mask=in_mask)

    def filter_mask(self, expr: str, values) -> np.ndarray:
        """Host values in, host u64 mask out (filter_jit.rs:71-121)."""
        torch = _torch()
        v = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float64)).to(_dev(self.device))
        m = self.filter_mask_gpu(expr, v)
        return _to_host_words(m)


class MaskOp:
    """MaskOp (filter_jit.rs:262-440): bitwise algebra of packed u64 row masks on the device."""

    def __init__(self, device: int = 0):
        self.device = device
        self.ctx = _ctx(device)

    # device-resident masks
    def mask_and_gpu(self, a, b, n_words: int):
        return self.ctx.mask_and(a[:n_words], b[:n_words])

    def mask_or_gpu(self, a, b, n_words: int):
        return self.ctx.mask_or(a[:n_words], b[:n_words])

    def mask_xor_gpu(self, a, b, n_words: int):
        return self.ctx.mask_xor(a[:n_words], b[:n_words])

    def mask_not_gpu(self, a, n_words: int, n_rows: int):
        return self.ctx.mask_not(a[:n_words], n_rows)

    def mask_popcount_gpu(self, mask, n_words: int, n_rows: int) -> int:
        return self.ctx.mask_popcount(mask[:n_words], n_rows)

    # host wrappers (upload, compute on the device, download)
    def _binary(self, fn, a, b):
        a = np.asarray(a, dtype=np.uint64)
        b = np.asarray(b, dtype=np.uint64)
        if a.size != b.size:
            raise InvalidArgument(7, "mask length mismatch")
        return _to_host_words(fn(_to_device_words(a, self.device), _to_device_words(b, self.device), a.size))

    def mask_and(self, a, b) -> np.ndarray:
        return self._binary(self.mask_and_gpu, a, b)

    def mask_or(self, a, b) -> np.ndarray:
        return self._binary(self.mask_or_gpu, a, b)

    def mask_xor(self, a, b) -> np.ndarray:
        return self._binary(self.mask_xor_gpu, a, b)

    def mask_not(self, mask, n_rows: int) -> np.ndarray:
        m = np.asarray(mask, dtype=np.uint64)
        return _to_host_words(self.mask_not_gpu(_to_device_words(m, self.device), m.size, n_rows))


# ---- .tb tile statistics (format.rs:60-189) ----

def tile_stats_numpy(stats) -> np.ndarray:
    """A device stats tensor [n_tiles, 40] as a host structured array (TileColumnStats fields)."""
    raw = stats.cpu().numpy()
    return np.ascontiguousarray(raw).view(TILE_STATS_DTYPE).reshape(-1)


def tile_skip_mask_gt(stats, threshold: float, device: int = 0):
    """tile_skip_mask_gt (format.rs:182-184): 1 for tiles whose max <= threshold."""
    return _ctx(device).tile_skip_mask(stats, ">", threshold)


def tile_skip_mask_lt(stats, threshold: float, device: int = 0):
    """tile_skip_mask_lt (format.rs:187-189): 1 for tiles whose min >= threshold."""
    return _ctx(device).tile_skip_mask(stats, "<", threshold)


def _fmin(a, b):
    return b if a != a else (a if b != b else (a if a < b else b))


def _fmax(a, b):
    return b if a != a else (a if b != b else (a if a > b else b))


def global_min(stats) -> float:
    """global_min (format.rs:144-149): over tiles with n_valid > 0, header only."""
    s = tile_stats_numpy(stats)
    out = math.inf
    for t in s[s["n_valid"] > 0]:
        out = _fmin(out, float(t["min"]))
    return out


def global_max(stats) -> float:
    """global_max (format.rs:152-157)."""
    s = tile_stats_numpy(stats)
    out = -math.inf
    for t in s[s["n_valid"] > 0]:
        out = _fmax(out, float(t["max"]))
    return out


def global_sum(stats) -> float:
    """global_sum (format.rs:160-162): sequential sum of the tile sums."""
    out = 0.0
    for v in tile_stats_numpy(stats)["sum"]:
        out += float(v)
    return out


def global_count(stats) -> int:
    """global_count (format.rs:165-167)."""
    return int(tile_stats_numpy(stats)["count"].astype(np.uint64).sum())


def global_mean(stats) -> float:
    """global_mean (format.rs:171-174)."""
    c = global_count(stats)
    return math.nan if c == 0 else global_sum(stats) / c


# ---- the Python caller surface (crates/tambear-py/src/lib.rs) ----

@dataclass
class GroupByResult(_OneScanResult):
    """GroupByResult (tambear-py lib.rs:72-135): sums, sum_sqs, counts per group.  ``m2``
    (sum of squared deviations from the group mean, from the fused one-pass kernel) is kept
    too, and ``variances()`` uses it: m2 / (count - 1), free of the cancellation of the
    sum_sqs - sums^2 / count formula; ``sum_sqs`` is m2 + sums^2 / count."""

    m2: np.ndarray | None = None

    def variances(self) -> np.ndarray:
        if self.m2 is None:
            return super().variances()
        c = self.counts
        with np.errstate(invalid="ignore", divide="ignore"):
            return np.where(c > 1, self.m2 / np.where(c > 1, c - 1.0, 1.0), np.nan)

    def n_active(self) -> int:
        return int(np.count_nonzero(self.counts > 0))

    def __repr__(self) -> str:
        return f"GroupByResult(n_groups={self.n_groups}, n_active={self.n_active()})"


class GroupByBuilder:
    """GroupByBuilder (tambear-py lib.rs:139-221): ``frame.groupby(key).sum / mean / stats``.
    Rows outside the frame's row mask take no part."""

    def __init__(self, frame: "Frame", key_col: str, n_groups: int):
        self.frame = frame
        self.key_col = key_col
        self.n_groups = int(n_groups)

    def _run(self, val_col: str, fields) -> dict:
        f = self.frame
        keys = f._key(self.key_col)
        vals = f._values(val_col)
        if self.n_groups == 0:
            return {k: np.zeros(0) for k in fields}
        out = f.ctx.groupby_dense(keys, vals, self.n_groups, mask=f.row_mask, out=f.ctx.alloc_moments(self.n_groups, fields))
        return {k: v.cpu().numpy() for k, v in out.items()}

    def sum(self, val_col: str) -> GroupByResult:
        """Sum per group (counts and sum_sqs zero, as the reference's sum-only result)."""
        r = self._run(val_col, ("sum",))
        z = np.zeros(self.n_groups)
        return GroupByResult(self.n_groups, r["sum"], z, z.copy())

    def stats(self, val_col: str) -> GroupByResult:
        """Sum + count + mean + variance in one pass."""
        r = self._run(val_col, ("count", "sum", "m2"))
        c, s, m2 = r["count"], r["sum"], r["m2"]
        with np.errstate(invalid="ignore", divide="ignore"):
            sq = np.where(c > 0, m2 + s * s / np.where(c > 0, c, 1.0), 0.0)
        return GroupByResult(self.n_groups, s, sq, c, m2=m2)

    def mean(self, val_col: str) -> GroupByResult:
        return self.stats(val_col)

    def __repr__(self) -> str:
        return f"GroupByBuilder(key='{self.key_col}', n_groups={self.n_groups})"


@dataclass
class Frame:
    """A device-resident frame (tambear-py PyFrame, lib.rs:227-272, with the core Frame's
    row_mask, frame.rs:86-125).  ``row_mask`` is None (every row) or ceil(n_rows / 64)
    device words; ``filter`` returns a Frame sharing the columns with the mask narrowed."""

    n_rows: int
    columns_: dict
    column_names: list
    device: int = 0
    row_mask: object = None
    tile_rows: int = TB_TILE_SIZE_DEFAULT
    tile_stats_: dict = field(default_factory=dict)
    group_indices: dict = field(default_factory=dict)

    @property
    def ctx(self) -> Context:
        return _ctx(self.device)

    @property
    def columns(self) -> list:
        return list(self.column_names)

    def __len__(self) -> int:
        return self.n_rows

    def __repr__(self) -> str:
        return f"Frame(n_rows={self.n_rows}, columns={self.column_names})"

    def col(self, name: str):
        if name not in self.columns_:
            raise KeyError(f"column '{name}' not found")
        return self.columns_[name]

    def _key(self, name: str):
        torch = _torch()
        c = self.col(name)
        if c.dtype != torch.int32:
            raise TypeError("expected integer column for groupby key")
        return c

    def _values(self, name: str):
        torch = _torch()
        c = self.col(name)
        if c.dtype != torch.float64:
            raise TypeError(f"expected float column for values (got {c.numel()} ints)")
        return c

    def mask_word_count(self) -> int:
        return (self.n_rows + 63) // 64

    def is_filtered(self) -> bool:
        return self.row_mask is not None

    def active_rows(self) -> int:
        return self.n_rows if self.row_mask is None else self.ctx.mask_popcount(self.row_mask, self.n_rows)

    def groupby(self, key_col: str) -> GroupByBuilder:
        """n_groups = max key + 1 over the whole column, as the reference computes it."""
        keys = self._key(key_col)
        n_groups = int(keys.max().item()) + 1 if self.n_rows else 0
        return GroupByBuilder(self, key_col, max(n_groups, 0))

    def tile_stats(self, col: str):
        """Per-tile TileColumnStats of a value column (built once, like a .tb header)."""
        if col not in self.tile_stats_:
            self.tile_stats_[col] = self.ctx.tile_stats(self._values(col), self.tile_rows)
        return self.tile_stats_[col]

    def filter(self, col: str, expr: str, skip_tiles: bool = True) -> "Frame":
        """Mask-not-filter: a Frame with the same columns and row_mask = row_mask AND expr(col).
        For a comparison, tiles whose statistics rule every row out are cleared first and the
        predicate then reads only the remaining tiles."""
        pred, thr = parse_predicate(expr)
        vals = self._values(col)
        base = self.row_mask
        if skip_tiles and pred in (">", ">=", "<", "<="):
            skip = self.ctx.tile_skip_mask(self.tile_stats(col), pred, thr)
            base = self.ctx.mask_skip_tiles(skip, self.tile_rows, self.n_rows, mask=base)
        m = self.ctx.filter_mask(vals, pred, thr, in_mask=base, out=base if base is not self.row_mask else None)
        return Frame(self.n_rows, self.columns_, self.column_names, self.device, m, self.tile_rows,
                     self.tile_stats_, self.group_indices)

    def group_index_for(self, key_col: str, max_key: int):
        """Frame::group_index_for (frame.rs:139-159): build the GroupIndex once per key column,
        rebuilt when the column's storage changed (provenance = data pointer + version)."""
        from .group_index import GroupIndex

        c = self._key(key_col)
        tag = (c.data_ptr(), c._version, int(max_key))
        hit = self.group_indices.get(key_col)
        if hit is not None and hit[0] == tag:
            return hit[1]
        gi = GroupIndex.build(self.ctx, c, int(max_key))
        self.group_indices[key_col] = (tag, gi)
        return gi


def from_columns(data: dict, device: int = 0) -> Frame:
    """from_columns (tambear-py lib.rs:286-329): integer columns become int32 key columns,
    float columns f64 value columns; all columns must have the same length."""
    torch = _torch()
    cols, names, n_rows = {}, [], None
    for name, values in data.items():
        if isinstance(values, torch.Tensor):
            t = values
        else:
            arr = np.asarray(values)
            if arr.dtype.kind in "iub" and arr.size and arr.min() >= -(2 ** 31) and arr.max() < 2 ** 31:
                arr = arr.astype(np.int32)
            elif arr.dtype.kind in "iub" and arr.size == 0:
                arr = arr.astype(np.int32)
            else:
                arr = arr.astype(np.float64)
            t = torch.from_numpy(np.ascontiguousarray(arr))
        if t.dtype not in (torch.int32, torch.float64):
            t = t.to(torch.int32 if not t.is_floating_point() else torch.float64)
        n = int(t.numel())
        if n_rows is not None and n != n_rows:
            raise ValueError(f"column '{name}' has {n} rows, expected {n_rows}")
        n_rows = n
        cols[name] = t.to(_dev(device)).contiguous()
        names.append(name)
    return Frame(n_rows or 0, cols, names, device)
