"""GPU parity of the scatter primitives (tbgb_scatter_* through ComputeEngine /
AccumulateEngine / HashScatterEngine) against the reference's golden vectors and the oracle.
Sums: |got - want| <= 1e-12 * sum|phi| over the finite terms; extrema bit-exact."""
import json
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from parity import bits

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402

CASES = json.loads((GOLDEN / "reference_vectors.json").read_text())["cases"]
ALL_PHIS = ["v", "v * v", "1.0", "v - r", "(v - r) * (v - r)", "fabs(v - r)", "(v - r) * (v - r) * (v - r)",
            "(v - r) * (v - r) * (v - r) * (v - r)", "v * r", "log(v)", "1.0 / v"]


@pytest.fixture(scope="module")
def eng():
    import winrapids_b200 as wb

    return wb.ComputeEngine(0)


def dec(x):
    return float(x) if x in ("nan", "inf", "-inf") else float.fromhex(x)


def phi_abs(phi, keys, vals, refs, G, mask_rows=None):
    """sum over rows of |phi| (finite terms) per group: the tolerance scale."""
    r = np.zeros(G) if refs is None else np.asarray(refs, np.float64)
    v = np.asarray(vals, np.float64)
    rk = r[np.asarray(keys)]
    with np.errstate(all="ignore"):
        t = {"v": v, "v * v": v * v, "1.0": np.ones_like(v), "v - r": v - rk, "(v - r) * (v - r)": (v - rk) ** 2,
             "fabs(v - r)": np.abs(v - rk), "(v - r) * (v - r) * (v - r)": (v - rk) ** 3,
             "(v - r) * (v - r) * (v - r) * (v - r)": (v - rk) ** 4, "v * r": v * rk, "log(v)": np.log(v),
             "1.0 / v": 1.0 / v}[phi]
    ok = np.isfinite(t)
    if mask_rows is not None:
        ok &= mask_rows
    return np.bincount(np.asarray(keys)[ok], weights=np.abs(t[ok]), minlength=G)


def close(got, want, scale):
    return np.all(np.abs(np.asarray(got) - np.asarray(want)) <= 1e-12 * scale + 0.0)


# ---- golden vectors ----------------------------------------------------------------------

@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "scatter_phi"], ids=lambda c: c["cite"])
def test_golden_scatter_phi(eng, case):
    keys, vals = make_golden.case_inputs(case)
    refs = None if "refs" not in case else np.array([dec(r) for r in case["refs"]])
    G = case["n_groups"]
    got = eng.scatter_phi(case["phi"], keys, vals, refs, G)
    want = np.array([dec(e) for e in case["expect"]])
    assert close(got, want, phi_abs(case["phi"], keys, vals, refs, G)), (got, want)


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "scatter_multi_phi"], ids=lambda c: c["cite"])
def test_golden_scatter_multi_phi(eng, case):
    keys, vals = make_golden.case_inputs(case)
    G = case["n_groups"]
    got = eng.scatter_multi_phi(case["phis"], keys, vals, None, G)
    for phi, g, exp in zip(case["phis"], got, case["expect"]):
        assert close(g, [dec(e) for e in exp], phi_abs(phi, keys, vals, None, G)), (phi, g, exp)


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "scatter_phi_masked"], ids=lambda c: c["cite"])
def test_golden_scatter_phi_masked(eng, case):
    keys, vals = make_golden.case_inputs(case)
    mask = np.array([int(w) for w in case["mask"]], dtype=np.uint64)
    G = case["n_groups"]
    got = eng.scatter_phi_masked(case["phi"], keys, vals, None, mask, G)
    n = len(keys)
    rows = ((mask[np.arange(n) // 64] >> (np.arange(n) % 64).astype(np.uint64)) & np.uint64(1)).astype(bool)
    want = [dec(e) for e in case["expect"]]
    assert close(got, want, phi_abs(case["phi"], keys, vals, None, G, rows)), (got, want)
    assert not np.any(np.signbit(got[np.asarray(want) == 0.0])), "empty masked sums are +0.0"


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "extremum"], ids=lambda c: c["cite"])
def test_golden_extremum(eng, case):
    keys, vals = make_golden.case_inputs(case)
    G = case["n_groups"]
    assert np.array_equal(bits(eng.scatter_extremum(False, keys, vals, G)), bits([dec(x) for x in case["expect_min"]]))
    assert np.array_equal(bits(eng.scatter_extremum(True, keys, vals, G)), bits([dec(x) for x in case["expect_max"]]))


def test_golden_unsupported_phi(eng):
    import winrapids_b200 as wb

    (case,) = [c for c in CASES if c["kind"] == "unsupported_phi"]
    with pytest.raises(wb.TambearGbError) as ei:
        eng.scatter_phi(case["phi"], [0], [1.0], None, 1)
    assert ei.value.kind == "EntryNotFound"


# ---- every phi, both accumulation paths, against the oracle --------------------------------

@pytest.mark.parametrize("G", [7, 3000, 40000])
def test_all_phis_vs_oracle(eng, G):
    rng = np.random.default_rng(G)
    n = 400_000
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = rng.normal(2.0, 1.5, n)
    vals[rng.random(n) < 0.01] = np.nan
    vals[rng.random(n) < 0.005] = np.inf
    vals[rng.random(n) < 0.01] = 0.0
    refs = rng.normal(2.0, 0.5, G)
    for start in range(0, len(ALL_PHIS), 5):
        phis = ALL_PHIS[start:start + 5]
        got = eng.scatter_multi_phi(phis, keys, vals, refs, G)
        want = oracle.scatter_multi_phi(phis, keys, vals, refs, G)
        for phi, g, w in zip(phis, got, want):
            assert close(g, w, phi_abs(phi, keys, vals, refs, G)), phi


def test_masked_multi_vs_oracle(eng):
    rng = np.random.default_rng(3)
    n, G = 300_001, 500
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = rng.normal(size=n)
    mask = rng.integers(0, 2**63, (n + 63) // 64, dtype=np.int64).astype(np.uint64)
    keys[5] = G + 3  # out of range but masked out: not an error
    mask[0] &= ~np.uint64(1 << 5)
    got = eng.scatter_multi_phi_masked(["v", "v * v", "1.0"], keys, vals, None, mask, G)
    rows = ((mask[np.arange(n) // 64] >> (np.arange(n) % 64).astype(np.uint64)) & np.uint64(1)).astype(bool)
    for phi, g in zip(["v", "v * v", "1.0"], got):
        w = oracle.scatter_phi_masked(phi, keys, vals, None, mask, G)
        assert close(g, w, phi_abs(phi, np.where(rows, keys, 0), vals, None, G, rows)), phi


@pytest.mark.parametrize("G", [1, 64, 5000])
def test_extremum_vs_oracle(eng, G):
    rng = np.random.default_rng(G + 1)
    n = 500_000
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = np.where(rng.random(n) < 0.5, 0.0, -0.0) * (rng.random(n) < 0.9) + rng.normal(size=n) * (rng.random(n) < 0.1)
    vals[rng.random(n) < 0.05] = np.nan
    for is_max in (False, True):
        got = eng.scatter_extremum(is_max, keys, vals, G)
        want = oracle.scatter_extremum(is_max, keys, vals, G)
        assert np.array_equal(bits(got), bits(want)), is_max


def test_key_out_of_range(eng):
    import winrapids_b200 as wb

    with pytest.raises(wb.KeyOutOfRange):
        eng.scatter_phi("v", [0, 5], [1.0, 2.0], None, 3)
    with pytest.raises(wb.KeyOutOfRange):
        eng.scatter_extremum(True, [0, -1], [1.0, 2.0], 3)
    assert eng.scatter_phi("v", [0, 1], [1.0, 2.0], None, 2).tolist() == [1.0, 2.0]


# ---- AccumulateEngine / HashScatterEngine ----------------------------------------------------

def test_accumulate_engine_matches_oracle():
    import winrapids_b200 as wb

    acc = wb.AccumulateEngine(0)
    rng = np.random.default_rng(5)
    n, G = 100_000, 37
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = rng.normal(size=n)
    mask = rng.integers(0, 2**63, (n + 63) // 64, dtype=np.int64).astype(np.uint64)
    absum = np.bincount(keys, weights=np.abs(vals), minlength=G)
    s = acc.accumulate(vals, wb.Grouping.All(), "v", wb.Op.Add)
    assert abs(s - oracle.exact_sum(vals)) <= 1e-12 * np.abs(vals).sum()
    assert acc.accumulate(vals, wb.Grouping.All(), "v", wb.Op.Max) == vals.max()
    assert acc.accumulate(vals, wb.Grouping.All(), "v", wb.Op.Min) == vals.min()
    by = wb.Grouping.ByKey(keys, G)
    assert close(acc.accumulate(vals, by, "v", wb.Op.Add), oracle.scatter_phi("v", keys, vals, None, G), absum)
    assert np.array_equal(acc.accumulate(vals, by, "v", wb.Op.Max), oracle.scatter_extremum(True, keys, vals, G))
    assert np.array_equal(acc.accumulate(vals, by, "v", wb.Op.Min), oracle.scatter_extremum(False, keys, vals, G))
    mk = wb.Grouping.Masked(keys, G, mask)
    assert close(acc.accumulate(vals, mk, "v", wb.Op.Add), oracle.scatter_phi_masked("v", keys, vals, None, mask, G),
                 absum)
    multi = acc.accumulate_multi(vals, by, ["v", "1.0"])
    assert np.array_equal(multi[1], np.bincount(keys, minlength=G).astype(float))
    mm = acc.accumulate_multi(vals, mk, ["v", "1.0"])
    assert close(mm[0], oracle.scatter_phi_masked("v", keys, vals, None, mask, G), absum)
    with pytest.raises(wb.TambearGbError):
        acc.accumulate(vals, mk, "v", wb.Op.Max)


def test_hash_scatter_engine_groupby():
    import winrapids_b200 as wb

    hs = wb.HashScatterEngine(0)
    rng = np.random.default_rng(9)
    n, G = 200_000, 4600
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = rng.normal(size=n)
    r = hs.groupby(keys, vals, G)
    absum = np.bincount(keys, weights=np.abs(vals), minlength=G)
    assert close(r.sums, oracle.scatter_phi("v", keys, vals, None, G), absum)
    assert close(r.sum_sqs, oracle.scatter_phi("v * v", keys, vals, None, G),
                 np.bincount(keys, weights=vals * vals, minlength=G))
    assert np.array_equal(r.counts, np.bincount(keys, minlength=G).astype(float))
    assert np.allclose(r.means(), r.sums / r.counts)
    assert np.array_equal(hs.value_counts(keys, G), r.counts)
    assert close(hs.scatter_sum(keys, vals, G), r.sums, absum)
