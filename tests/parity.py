"""Shared parity checks: GPU outputs vs the oracle, with the tolerances of the
groupby contract:
  count, min, max        bit-exact (min/max compared as bit patterns, so +-0 matters)
  sum                    |got - want| <= 1e-12 * sum(|x|) over the group's finite values
  mean                   |got - want| <= 1e-12 * sum(|x|) / count
  m2, var_pop, var_samp  |got - want| <= 1e-9 * |want|, NaN exactly where the oracle has NaN
"""
from __future__ import annotations

import numpy as np

SUM_TOL = 1e-12
VAR_RTOL = 1e-9


def abs_sums(keys, vals, n_groups, mask_rows=None):
    v = np.asarray(vals, dtype=np.float64)
    k = np.asarray(keys)
    fin = np.isfinite(v)
    if mask_rows is not None:
        fin &= mask_rows
    return np.bincount(k[fin], weights=np.abs(v[fin]), minlength=n_groups)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float64).view(np.uint64)


def check(got: dict, want: dict, absum: np.ndarray, label: str = ""):
    """got: {count,sum,min,max,mean,m2,var_pop,var_samp} numpy; want: oracle moments + derived."""
    import oracle

    d = oracle.derived(want)
    c = want["counts"]
    assert np.array_equal(got["count"], c), f"{label} count"
    assert np.array_equal(bits(got["min"]), bits(want["mins"])), f"{label} min bits"
    assert np.array_equal(bits(got["max"]), bits(want["maxs"])), f"{label} max bits"
    err = np.abs(got["sum"] - want["sums"])
    assert np.all(err <= SUM_TOL * absum), f"{label} sum err {np.max(err - SUM_TOL * absum)}"
    cnt = np.where(c > 0, c, 1.0)
    m_ok = np.where(c > 0, np.abs(got["mean"] - d["mean"]) <= SUM_TOL * absum / cnt, np.isnan(got["mean"]))
    assert np.all(m_ok), f"{label} mean"
    for f, w in (("m2", want["m2s"]), ("var_pop", d["var_pop"]), ("var_samp", d["var_samp"])):
        g = got[f]
        nan_w = np.isnan(w)
        assert np.array_equal(np.isnan(g), nan_w), f"{label} {f} NaN pattern"
        ww, gg = w[~nan_w], g[~nan_w]
        assert np.all(np.abs(gg - ww) <= VAR_RTOL * np.abs(ww)), \
            f"{label} {f} rel err {np.max(np.abs(gg - ww) / np.maximum(np.abs(ww), 1e-300))}"


def to_host(out: dict) -> dict:
    return {k: v.detach().cpu().numpy() for k, v in out.items()}
