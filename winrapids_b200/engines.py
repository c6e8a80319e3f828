"""The reference's scatter-level operator API over the B200 kernels (host slices in, host
arrays out, like the reference's `&[T]` -> `Vec<f64>` methods):

* ``ComputeEngine``      scatter_phi / scatter_multi_phi / scatter_phi_masked / scatter_extremum
                         (crates/tambear/src/compute_engine.rs:87-178)
* ``AccumulateEngine``   accumulate / accumulate_multi over Grouping.All / ByKey / Masked with
                         Op.Add / Max / Min (crates/tambear/src/accumulate.rs:43-70, 181, 638-790)
* ``HashScatterEngine``  scatter_sum / value_counts / groupby -> GroupByResult
                         (crates/tambear/src/hash_scatter.rs:176-230, 324-435)

Every call runs on the GPU through the C ABI; there is no CPU path.  Arithmetic follows
the reference's CPU backend: phi sums skip +-0 / NaN / +-inf terms, extrema are strict
scans with +-0 ties to the first zero.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import PHI_IDS, InvalidArgument, TambearGbError


def _phi_id(expr: str) -> int:
    key = " ".join(expr.split())
    if key not in PHI_IDS:
        raise TambearGbError(6, f"unknown phi expression {expr!r}")
    return PHI_IDS[key]


class ComputeEngine:
    """ComputeEngine (compute_engine.rs:87-178) on one B200."""

    def __init__(self, device: int = 0):
        from . import Context

        self.ctx = Context(device)
        self._dev = f"cuda:{device}"

    def _up(self, x, dtype):
        import torch

        return torch.as_tensor(np.ascontiguousarray(x, dtype=dtype)).to(self._dev)

    def _scatter(self, phis, keys, values, refs, mask, n_groups):
        import torch

        keys = np.asarray(keys)
        values = np.asarray(values)
        if keys.size != values.size:
            raise InvalidArgument(7, "keys and values must have same length")
        if refs is not None and np.asarray(refs).size != n_groups:
            raise InvalidArgument(7, "refs must have length n_groups")
        ids = (C.c_int32 * len(phis))(*[_phi_id(p) for p in phis])
        dk, dv = self._up(keys, np.int32), self._up(values, np.float64)
        dr = None if refs is None else self._up(refs, np.float64)
        dm = None if mask is None else self._up(np.asarray(mask, dtype=np.uint64).view(np.int64), np.int64)
        out = torch.empty(len(phis) * int(n_groups), dtype=torch.float64, device=self._dev)
        L, h = self.ctx._L, self.ctx._h
        st = L.tbgb_scatter_multi_phi_masked(h, ids, len(phis), dk.data_ptr(), dv.data_ptr(),
                                             None if dr is None else dr.data_ptr(),
                                             None if dm is None else dm.data_ptr(), keys.size, int(n_groups),
                                             out.data_ptr(), None)
        self.ctx._check(st)
        self.ctx.sync(0)
        return out.cpu().numpy().reshape(len(phis), int(n_groups))

    def scatter_phi(self, phi_expr: str, keys, values, refs=None, n_groups: int = 1) -> np.ndarray:
        """output[keys[i]] += phi(values[i], refs[keys[i]])."""
        return self._scatter([phi_expr], keys, values, refs, None, n_groups)[0]

    def scatter_multi_phi(self, phi_exprs, keys, values, refs=None, n_groups: int = 1) -> list[np.ndarray]:
        """Up to five phi expressions in one pass."""
        return list(self._scatter(list(phi_exprs), keys, values, refs, None, n_groups))

    def scatter_phi_masked(self, phi_expr: str, keys, values, refs, mask, n_groups: int) -> np.ndarray:
        """scatter_phi over the rows whose bit is set in mask (bit i of mask[i // 64])."""
        return self._scatter([phi_expr], keys, values, refs, mask, n_groups)[0]

    def scatter_multi_phi_masked(self, phi_exprs, keys, values, refs, mask, n_groups: int) -> list[np.ndarray]:
        """ScatterJit::scatter_multi_phi_masked (scatter_jit.rs:402-495): masked, one pass."""
        return list(self._scatter(list(phi_exprs), keys, values, refs, mask, n_groups))

    def scatter_extremum(self, is_max: bool, keys, values, n_groups: int) -> np.ndarray:
        """Per-group max (is_max) or min; +-inf for groups without a non-NaN value."""
        import torch

        keys = np.asarray(keys)
        values = np.asarray(values)
        if keys.size != values.size:
            raise InvalidArgument(7, "keys and values must have same length")
        dk, dv = self._up(keys, np.int32), self._up(values, np.float64)
        out = torch.empty(int(n_groups), dtype=torch.float64, device=self._dev)
        self.ctx._check(self.ctx._L.tbgb_scatter_extremum(self.ctx._h, 1 if is_max else 0, dk.data_ptr(),
                                                          dv.data_ptr(), keys.size, int(n_groups), out.data_ptr(),
                                                          None))
        self.ctx.sync(0)
        return out.cpu().numpy()


# ---- AccumulateEngine (accumulate.rs) --------------------------------------------------

@dataclass(frozen=True)
class All:
    """Grouping::All: one group."""


@dataclass(frozen=True)
class ByKey:
    """Grouping::ByKey { keys, n_groups }."""
    keys: object
    n_groups: int


@dataclass(frozen=True)
class Masked:
    """Grouping::Masked { keys, n_groups, mask }."""
    keys: object
    n_groups: int
    mask: object


class Grouping:
    All = All
    ByKey = ByKey
    Masked = Masked


class Op:
    """accumulate.rs:181 Op (the variants this path computes)."""
    Add = "add"
    Max = "max"
    Min = "min"


class AccumulateEngine:
    """AccumulateEngine::accumulate / accumulate_multi (accumulate.rs:638-790)."""

    def __init__(self, device: int = 0):
        self.compute = ComputeEngine(device)

    def accumulate(self, values, grouping, expr: str, op: str):
        """Returns a float for Grouping.All (AccResult::Scalar), else a per-group array
        (AccResult::PerGroup)."""
        values = np.asarray(values, dtype=np.float64)
        if isinstance(grouping, All):
            keys = np.zeros(values.size, dtype=np.int32)
            if op == Op.Add:
                return float(self.compute.scatter_phi(expr, keys, values, None, 1)[0])
            if op in (Op.Max, Op.Min):
                return float(self.compute.scatter_extremum(op == Op.Max, keys, values, 1)[0])
        elif isinstance(grouping, ByKey):
            if op == Op.Add:
                return self.compute.scatter_phi(expr, grouping.keys, values, None, grouping.n_groups)
            if op in (Op.Max, Op.Min):
                return self.compute.scatter_extremum(op == Op.Max, grouping.keys, values, grouping.n_groups)
        elif isinstance(grouping, Masked):
            if op == Op.Add:
                return self.compute.scatter_phi_masked(expr, grouping.keys, values, None, grouping.mask,
                                                       grouping.n_groups)
        raise TambearGbError(7, "accumulate: unsupported (grouping, op) combination")

    def accumulate_multi(self, values, grouping, phi_exprs) -> list[np.ndarray]:
        """Several Add expressions over one grouping in one pass (the masked grouping is fused
        too, where the reference issues one masked scatter per expression)."""
        if isinstance(grouping, ByKey):
            return self.compute.scatter_multi_phi(phi_exprs, grouping.keys, values, None, grouping.n_groups)
        if isinstance(grouping, Masked):
            return self.compute.scatter_multi_phi_masked(phi_exprs, grouping.keys, values, None, grouping.mask,
                                                         grouping.n_groups)
        raise TambearGbError(7, "accumulate_multi: only ByKey and Masked groupings supported")


# ---- HashScatterEngine (hash_scatter.rs) -----------------------------------------------

@dataclass
class GroupByResult:
    """sum + sum of squares + count per group (hash_scatter.rs:176-230)."""
    n_groups: int
    sums: np.ndarray
    sum_sqs: np.ndarray
    counts: np.ndarray

    def means(self) -> np.ndarray:
        c = self.counts
        with np.errstate(invalid="ignore", divide="ignore"):
            return np.where(c > 0, self.sums / np.where(c > 0, c, 1.0), np.nan)

    def variances(self) -> np.ndarray:
        """The reference's one-pass formula (deprecated there for large offsets; the fused
        groupby's var_samp is the stable one)."""
        c, s, sq = self.counts, self.sums, self.sum_sqs
        with np.errstate(invalid="ignore", divide="ignore"):
            m = s / np.where(c > 0, c, 1.0)
            v = np.maximum((sq / np.where(c > 0, c, 1.0) - m * m) * c / np.where(c > 1, c - 1.0, 1.0), 0.0)
        return np.where(c > 1, v, np.nan)

    def stds(self) -> np.ndarray:
        return np.sqrt(self.variances())


class HashScatterEngine:
    """HashScatterEngine (hash_scatter.rs:270-435): dense int32 keys in [0, n_groups)."""

    def __init__(self, device: int = 0):
        self.compute = ComputeEngine(device)

    def scatter_sum(self, keys, values, n_groups: int) -> np.ndarray:
        return self.compute.scatter_phi("v", keys, values, None, n_groups)

    def value_counts(self, keys, n_groups: int) -> np.ndarray:
        keys = np.asarray(keys)
        return self.compute.scatter_phi("1.0", keys, np.zeros(keys.size), None, n_groups)

    def groupby(self, keys, values, n_groups: int) -> GroupByResult:
        s, sq, c = self.compute.scatter_multi_phi(["v", "v * v", "1.0"], keys, values, None, n_groups)
        return GroupByResult(int(n_groups), s, sq, c)
