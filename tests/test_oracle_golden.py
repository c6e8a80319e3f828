"""Pin the oracle (C restatement of the reference's CPU groupby) to the reference's
own golden vectors (tests/golden/reference_vectors.json, each case cites its test).
CPU only."""
import json
import math
import struct
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402

CASES = json.loads((GOLDEN / "reference_vectors.json").read_text())["cases"]


def dec(x):
    if x is None:
        return None
    if isinstance(x, (int, float)):
        return float(x)
    return float(x) if x in ("nan", "inf", "-inf") else float.fromhex(x)


def bits(x: float) -> int:
    return struct.unpack("<Q", struct.pack("<d", x))[0]


def same(a, b, tol=0.0, rel=False):
    a, b = float(a), float(b)
    if math.isnan(b):
        return math.isnan(a)
    if tol == 0.0:
        return bits(a) == bits(b)
    err = abs(a - b)
    return err <= tol * (abs(b) if rel else 1.0)


def ids(kind):
    return [c for c in CASES if c["kind"] == kind]


@pytest.mark.parametrize("case", ids("exact_sum") + ids("exact_sum_tol"), ids=lambda c: c["cite"])
def test_exact_sum(case):
    _, vals = make_golden.case_inputs(case)
    got = oracle.exact_sum(np.array(vals))
    assert same(got, dec(case["expect"]), case.get("tol", 0.0)), (got, case["expect"])


@pytest.mark.parametrize("case", ids("scatter_phi"), ids=lambda c: c["cite"])
def test_scatter_phi(case):
    keys, vals = make_golden.case_inputs(case)
    refs = None if "refs" not in case else np.array([dec(r) for r in case["refs"]])
    got = oracle.scatter_phi(case["phi"], keys, vals, refs, case["n_groups"])
    for g, e in zip(got, case["expect"]):
        assert same(g, dec(e)), (list(got), case["expect"])


@pytest.mark.parametrize("case", ids("scatter_multi_phi"), ids=lambda c: c["cite"])
def test_scatter_multi_phi(case):
    keys, vals = make_golden.case_inputs(case)
    got = oracle.scatter_multi_phi(case["phis"], keys, vals, None, case["n_groups"])
    for out, exp in zip(got, case["expect"]):
        assert all(same(g, dec(e)) for g, e in zip(out, exp)), (got, case["expect"])


@pytest.mark.parametrize("case", ids("scatter_phi_masked"), ids=lambda c: c["cite"])
def test_scatter_phi_masked(case):
    keys, vals = make_golden.case_inputs(case)
    mask = np.array([int(w) for w in case["mask"]], dtype=np.uint64)
    got = oracle.scatter_phi_masked(case["phi"], keys, vals, None, mask, case["n_groups"])
    for g, e in zip(got, case["expect"]):
        assert same(g, dec(e)), (list(got), case["expect"])


@pytest.mark.parametrize("case", ids("extremum"), ids=lambda c: c["cite"])
def test_extremum(case):
    keys, vals = make_golden.case_inputs(case)
    mn = oracle.scatter_extremum(False, keys, vals, case["n_groups"])
    mx = oracle.scatter_extremum(True, keys, vals, case["n_groups"])
    assert all(same(a, dec(b)) for a, b in zip(mn, case["expect_min"]))
    assert all(same(a, dec(b)) for a, b in zip(mx, case["expect_max"]))


def test_unsupported_phi_errors():
    (case,) = ids("unsupported_phi")
    with pytest.raises(oracle.OracleError):
        oracle.scatter_phi(case["phi"], [0], [1.0], None, 1)


def _derived_check(mom, exp, tol, rel):
    d = oracle.derived(mom)
    table = {"count": mom["counts"], "sum": mom["sums"], "min": mom["mins"], "max": mom["maxs"],
             "mean": d["mean"], "var_pop": d["var_pop"], "var_samp": d["var_samp"]}
    for field, want in exp.items():
        for g, w in enumerate(want):
            if w is None:
                continue
            assert same(table[field][g], dec(w), tol, rel), (field, g, table[field][g], w)


@pytest.mark.parametrize("case", ids("moments_grouped"), ids=lambda c: c["cite"])
def test_moments_grouped(case):
    keys, vals = make_golden.case_inputs(case)
    mom = oracle.moments_grouped(vals, keys, case["n_groups"])
    _derived_check(mom, case["expect"], case.get("tol", 0.0), case.get("rel", False))


def test_mean_grouped():
    (case,) = ids("mean_grouped")
    keys, vals = make_golden.case_inputs(case)
    mom = oracle.moments_grouped(vals, keys, case["n_groups"])
    means = oracle.derived(mom)["mean"]
    assert np.allclose(means, case["expect"], atol=case["tol"], rtol=0)


def test_grouped_higher_moments():
    (case,) = ids("moments_grouped_m34")
    keys, vals = make_golden.case_inputs(case)
    mom = oracle.moments_grouped(vals, keys, case["n_groups"])
    n, m2, m3, m4 = mom["counts"][0], mom["m2s"][0], mom["m3s"][0], mom["m4s"][0]
    var = m2 / n
    g1 = (m3 / n) / (var * math.sqrt(var))           # MomentStats::skewness(bias=true), descriptive.rs:135-148
    raw = (m4 / n) / (var * var)                     # MomentStats::kurtosis(excess, bias=true), :157-175
    assert abs(g1 - case["expect_g0"]["skew_biased"]) < case["tol"]
    assert abs((raw - 3.0) - case["expect_g0"]["kurt_excess_biased"]) < case["tol"]


# ---- oracle self-consistency --------------------------------------------------------

def test_mt_matches_single_thread_bit_for_bit():
    rng = np.random.default_rng(7)
    n, G = 200_003, 37
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = rng.standard_normal(n) * 10.0 ** rng.integers(-30, 30, n)
    vals[rng.random(n) < 0.01] = np.nan
    vals[rng.random(n) < 0.002] = np.inf
    vals[rng.random(n) < 0.002] = -np.inf
    vals[:50] = 0.0
    vals[50:100] = -0.0
    a = oracle.moments_grouped(vals, keys, G, m34=False)
    for t in (1, 3, 8):
        b = oracle.moments_grouped_mt(vals, keys, G, threads=t)
        for f in ("counts", "sums", "mins", "maxs", "m2s"):
            assert np.array_equal(a[f].view(np.uint64), b[f].view(np.uint64)), (t, f)


def test_i64_factorised_path_matches_dense_path():
    rng = np.random.default_rng(11)
    n, G = 50_000, 101
    ids_ = rng.integers(0, G, n)
    salt = rng.integers(-2**62, 2**62, G)
    keys64 = salt[ids_]
    vals = rng.standard_normal(n)
    vals[rng.random(n) < 0.02] = np.nan
    r = oracle.groupby_i64(keys64, vals)
    order = np.argsort(salt)  # dense id of each sorted key
    d = oracle.moments_grouped(vals, ids_.astype(np.int32), G, m34=False)
    assert np.array_equal(r["keys"], salt[order])
    for f in ("counts", "sums", "mins", "maxs", "m2s"):
        assert np.array_equal(r[f].view(np.uint64), d[f][order].view(np.uint64)), f


def test_masked_moments_equal_moments_of_filtered_rows():
    rng = np.random.default_rng(3)
    n, G = 10_000, 13
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = rng.standard_normal(n)
    mask = oracle.filter_mask("gt", 0.0, rng.standard_normal(n))
    sel = np.array([(int(mask[i // 64]) >> (i % 64)) & 1 for i in range(n)], dtype=bool)
    a = oracle.moments_grouped_masked(vals, keys, mask, G)
    b = oracle.moments_grouped(vals[sel], keys[sel], G, m34=False)
    c = oracle.moments_grouped_mt(vals, keys, G, threads=4, mask=mask)
    for f in ("counts", "sums", "mins", "maxs", "m2s"):
        assert np.array_equal(a[f].view(np.uint64), b[f].view(np.uint64)), f
        assert np.array_equal(a[f].view(np.uint64), c[f].view(np.uint64)), f


def test_kulisch_matches_fsum_on_random_data():
    rng = np.random.default_rng(5)
    for _ in range(20):
        n = int(rng.integers(1, 5000))
        x = rng.standard_normal(n) * 10.0 ** rng.integers(-300, 300, n)
        assert bits(oracle.exact_sum(x)) == bits(math.fsum(x.tolist()) + 0.0)


def test_out_of_range_key_is_an_error():
    with pytest.raises(IndexError):
        oracle.moments_grouped([1.0, 2.0], [0, 5], 2)
    with pytest.raises(IndexError):
        oracle.moments_grouped([1.0, 2.0], [0, -1], 2)


def test_filter_mask_layout_and_map2():
    a = np.array([1.0, -1.0, np.nan, 0.0, 2.0] + [1.0] * 70)
    m = oracle.filter_mask("gt", 0.0, a)
    assert m.size == 2
    assert int(m[0]) & 0b11111 == 0b10001  # NaN fails a > 0
    assert int(m[1]) >> 11 == 0  # trailing bits of the last word stay 0
    b = np.array([2.0] * a.size)
    c = np.array([0.5] * a.size)
    ab = oracle.map2("a * b", a, b)
    v = oracle.map2("a + b", ab, c)
    assert v[0] == 2.5 and v[1] == -1.5


def test_generator_streams():
    # SplitMix64::new(seed).next_u64() sequence (rng.rs:73-83) == counter form
    seed = 0x1234
    state = seed
    seq = []
    for _ in range(5):
        state = (state + 0x9E3779B97F4A7C15) & oracle.M64
        seq.append(oracle.mix64_int(state))
    assert list(map(int, oracle.splitmix_stream(seed, 0, 5))) == seq
    assert [int(oracle.lib().orc_splitmix_at(seed, i)) for i in range(5)] == seq
    k = oracle.gen_keys_uniform(1000, 256, 0)
    assert k.min() >= 0 and k.max() < 256


def test_group_index_oracle_hand_case():
    """GroupIndex::build semantics (group_index.rs:117-204) on a hand-worked column: counts,
    offsets with the n sentinel, rows_by_group in row order inside each group."""
    gi = oracle.group_index_build([2, 0, 2, 1, 0], 3)
    assert gi["row_to_group"].tolist() == [2, 0, 2, 1, 0]
    assert gi["group_counts"].tolist() == [2, 1, 2, 0]
    assert gi["group_offsets"].tolist() == [0, 2, 3, 5, 5]
    assert gi["rows_by_group"].tolist() == [1, 4, 3, 0, 2]
    assert gi["n_active"] == 3


def test_factorize_oracle_first_seen_order():
    """Dictionary::encode (dictionary.rs:40-75): codes follow the order values are first seen."""
    codes, uniq = oracle.factorize_first_seen([5, 3, 5, -7, 3, 2**63 - 1, -(2**63)])
    assert codes.tolist() == [0, 1, 0, 2, 1, 3, 4]
    assert uniq.tolist() == [5, 3, -7, 2**63 - 1, -(2**63)]


# ---- mask-not-filter plumbing: FilterJit masks, mask algebra, tile statistics ----

def words(xs):
    return np.array([int(x, 16) for x in xs], dtype=np.uint64)


@pytest.mark.parametrize("case", ids("filter_mask"), ids=lambda c: c["cite"])
def test_filter_mask_golden(case):
    vals = [dec(v) for v in case["values"]]
    m = oracle.filter_mask(case["pred"], dec(case["threshold"]), vals)
    exp, chk = words(case["expect"]), words(case["check"])
    assert m.size == exp.size == (len(vals) + 63) // 64
    assert np.array_equal(m & chk, exp)


@pytest.mark.parametrize("case", ids("mask_binary"), ids=lambda c: c["cite"])
def test_mask_binary_golden(case):
    f = {"and": oracle.mask_and, "or": oracle.mask_or, "xor": oracle.mask_xor}[case["op"]]
    assert np.array_equal(f(words(case["a"]), words(case["b"])), words(case["expect"]))


@pytest.mark.parametrize("case", ids("mask_not"), ids=lambda c: c["cite"])
def test_mask_not_golden(case):
    out = oracle.mask_not(words(case["a"]), case["n_rows"])
    assert np.array_equal(out, words(case["expect"]))


@pytest.mark.parametrize("case", ids("mask_popcount") + ids("mask_and_popcount"), ids=lambda c: c["cite"])
def test_mask_popcount_golden(case):
    if case["kind"] == "mask_and_popcount":
        m = oracle.mask_and(words(case["a"]), words(case["b"]))
    else:
        m = words(case["mask"])
    assert oracle.mask_popcount(m, case["n_rows"]) == case["expect"]


@pytest.mark.parametrize("case", ids("tile_stats_global"), ids=lambda c: c["cite"])
def test_tile_stats_golden(case):
    vals = [float(i) for i in range(case["arange"])] if "arange" in case else [dec(v) for v in case["values"]]
    st = oracle.tile_stats(vals, case["tile_rows"])
    assert st.size == case["n_tiles"]
    g = oracle.tile_global_stats(st)
    e = case["expect"]
    assert same(g["min"], dec(e["min"])) and same(g["max"], dec(e["max"]))
    assert g["count"] == e["count"]
    assert abs(g["mean"] - dec(e["mean"])) < case["tol"]


def test_tile_stats_kahan_nonfinite():
    """The serial Kahan loop of TileColumnStats::from_slice: NaN anywhere -> NaN; an infinity
    followed by any value -> NaN; a single infinity as the tile's last value -> that infinity."""
    inf, nan = math.inf, math.nan
    st = oracle.tile_stats([1.0, 2.0, inf, 3.0, 1.0, 2.0, 3.0, -inf, 7.0, nan, -0.0, 0.0], 4)
    assert math.isnan(st["sum"][0])                 # inf then 3.0
    assert st["sum"][1] == -inf                     # -inf last
    assert math.isnan(st["sum"][2])                 # NaN
    assert st["min"][2] == 0.0 and math.copysign(1.0, st["min"][2]) == -1.0  # first zero (-0.0) kept
    assert st["max"][2] == 7.0
    allnan = oracle.tile_stats([nan, nan], 2)
    assert allnan["min"][0] == inf and allnan["max"][0] == -inf


def test_tile_skip_rules():
    st = oracle.tile_stats([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], 2)   # tiles [1,2] [3,4] [5,6]
    assert list(oracle.tile_skip(st, "gt", 4.0)) == [1, 1, 0]    # max <= 4
    assert list(oracle.tile_skip(st, "ge", 4.0)) == [1, 0, 0]    # max < 4
    assert list(oracle.tile_skip(st, "lt", 3.0)) == [0, 1, 1]    # min >= 3
    assert list(oracle.tile_skip(st, "le", 3.0)) == [0, 0, 1]    # min > 3
    assert list(oracle.tile_skip(st, "gt", math.nan)) == [0, 0, 0]


def test_bin_stats_restatement_hand_case():
    """fused_bin_stats (bin_stats.cu:25-77) on a hand case: an empty bin is NaN with count 0, a
    NaN first value is the bin's min and max, and the serial scan keeps the first of +-0."""
    r = oracle.bin_stats([1.0, 2.0, 3.0, math.nan, 5.0, -0.0, 0.0, 7.0], [0, 3, 3, 5, 8])
    assert list(r["count"]) == [3, 0, 2, 3]
    assert r["sum"][0] == 6.0 and r["sum_sq"][0] == 14.0 and r["min"][0] == 1.0 and r["max"][0] == 3.0
    assert all(math.isnan(r[k][1]) for k in ("sum", "sum_sq", "min", "max", "first", "last", "mean", "variance"))
    assert math.isnan(r["min"][2]) and math.isnan(r["max"][2]) and r["last"][2] == 5.0
    assert r["min"][3] == 0.0 and math.copysign(1.0, r["min"][3]) == -1.0 and r["max"][3] == 7.0
    assert r["first"][3] == 0.0 and math.copysign(1.0, r["first"][3]) == -1.0
