"""The host-side MomentStats mirror (descriptive.rs:67-254): derived statistics and the
parallel merge, on CPU (no GPU involved)."""
import math

import numpy as np
import pytest
from scipy import stats

import winrapids_b200 as wb


def ms(x):
    x = np.asarray(x, dtype=np.float64)
    m = x.mean()
    return wb.MomentStats(float(x.size), float(x.sum()), float(x.min()), float(x.max()),
                          float(((x - m) ** 2).sum()), float(((x - m) ** 3).sum()), float(((x - m) ** 4).sum()))


def test_derived_statistics_match_scipy():
    x = np.random.default_rng(0).lognormal(size=1000)
    s = ms(x)
    assert math.isclose(s.mean(), x.mean(), rel_tol=1e-12)
    assert math.isclose(s.variance(1), x.var(ddof=1), rel_tol=1e-12)
    assert math.isclose(s.skewness(True), stats.skew(x, bias=True), rel_tol=1e-10)
    assert math.isclose(s.skewness(False), stats.skew(x, bias=False), rel_tol=1e-10)
    assert math.isclose(s.kurtosis(True, True), stats.kurtosis(x, fisher=True, bias=True), rel_tol=1e-10)
    assert math.isclose(s.kurtosis(True, False), stats.kurtosis(x, fisher=True, bias=False), rel_tol=1e-10)
    assert math.isclose(s.kurtosis(False, False), stats.kurtosis(x, fisher=False, bias=False), rel_tol=1e-10)
    assert math.isclose(s.sem(), stats.sem(x), rel_tol=1e-12)


@pytest.mark.parametrize("split", [1, 17, 500, 999])
def test_merge_equals_whole(split):
    x = np.random.default_rng(split).normal(3.0, 2.0, 1000) ** 3
    m = wb.MomentStats.merge(ms(x[:split]), ms(x[split:]))
    w = ms(x)
    for f in ("count", "sum", "min", "max"):
        assert math.isclose(getattr(m, f), getattr(w, f), rel_tol=1e-12)
    for f in ("m2", "m3", "m4"):
        assert math.isclose(getattr(m, f), getattr(w, f), rel_tol=1e-8), f


def test_empty_and_small():
    e = wb.MomentStats.empty()
    assert math.isnan(e.mean()) and math.isnan(e.variance(0)) and math.isnan(e.skewness(True))
    assert wb.MomentStats.merge(e, ms([1.0, 2.0])).count == 2
    assert math.isnan(ms([1.0, 2.0]).skewness(False)) and math.isnan(ms([1.0, 2.0, 3.0]).kurtosis(True, False))
