"""GPU parity of the dense-key groupby (tbgb_groupby_dense, through the C ABI) against the oracle."""
import json
import math
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from parity import abs_sums, bits, check, to_host

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402

CASES = json.loads((GOLDEN / "reference_vectors.json").read_text())["cases"]


def run_gpu(ctx, keys, vals, G, mask=None):
    import torch

    dk = torch.as_tensor(np.ascontiguousarray(keys, dtype=np.int32)).cuda()
    dv = torch.as_tensor(np.ascontiguousarray(vals, dtype=np.float64)).cuda()
    dm = None if mask is None else torch.as_tensor(np.ascontiguousarray(mask, dtype=np.uint64).view(np.int64)).cuda()
    return to_host(ctx.groupby_dense(dk, dv, G, mask=dm))


def parity(ctx, keys, vals, G, label=""):
    got = run_gpu(ctx, keys, vals, G)
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8)
    check(got, want, abs_sums(keys, vals, G), label)
    return got, want


# ---- the reference's golden vectors --------------------------------------------------

@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "moments_grouped"], ids=lambda c: c["cite"])
def test_golden_moments(ctx, case):
    keys, vals = make_golden.case_inputs(case)
    got = run_gpu(ctx, keys, vals, case["n_groups"])
    table = {"count": got["count"], "mean": got["mean"], "min": got["min"], "max": got["max"],
             "var_pop": got["var_pop"], "var_samp": got["var_samp"], "sum": got["sum"]}
    tol, rel = case.get("tol", 0.0), case.get("rel", False)
    for field, want in case["expect"].items():
        for g, w in enumerate(want):
            if w is None:
                continue
            w = float(w) if not isinstance(w, str) else float(w)
            a = table[field][g]
            if math.isnan(w):
                assert math.isnan(a), (field, g)
            elif math.isinf(w):
                assert a == w, (field, g, a, w)
            else:
                assert abs(a - w) <= (tol * (abs(w) if rel else 1.0)), (field, g, a, w)


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] in ("extremum", "scatter_phi")
                                  and c.get("phi", "v") == "v" and "refs" not in c], ids=lambda c: c["cite"])
def test_golden_sum_and_extrema(ctx, case):
    keys, vals = make_golden.case_inputs(case)
    G = case["n_groups"]
    got = run_gpu(ctx, keys, vals, G)
    absum = abs_sums(keys, vals, G)
    if case["kind"] == "extremum":
        assert np.array_equal(bits(got["min"]), bits([float.fromhex(x) for x in case["expect_min"]]))
        assert np.array_equal(bits(got["max"]), bits([float.fromhex(x) for x in case["expect_max"]]))
    else:
        want = np.array([float.fromhex(x) for x in case["expect"]])
        assert np.all(np.abs(got["sum"] - want) <= 1e-12 * absum), (got["sum"], want)


# ---- the configurations' shapes at oracle-friendly sizes ------------------------------

def test_config1_full(ctx):
    """1,000,000 rows, int32 keys in [0,1000), f64 ~N(0,1), seed 0: the reference's CPU-runnable config."""
    n, G = 1_000_000, 1000
    keys = oracle.gen_keys_uniform(n, G, 0)
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 0)
    parity(ctx, keys, vals, G, "C1")


def test_low_cardinality_uniform(ctx):
    n, G = 3_000_017, 256
    keys = oracle.gen_keys_uniform(n, G, 3)
    vals = oracle.gen_values_uniform(n, -1.0, 1.0, 3)
    parity(ctx, keys, vals, G, "C3-shape")


def test_numerical_stress_shape(ctx):
    """1e9 + N(0, 1e-3) with 1% NaN and 0.1% +-inf (the stress config's value model)."""
    n, G = 2_000_000, 1000
    keys = oracle.gen_keys_uniform(n, G, 5)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 1e9, 1e-3, 5), 0.01, 0.001, 5)
    parity(ctx, keys, vals, G, "C5-shape")


def test_stress_without_inf_variance_is_tight(ctx):
    n, G = 1_000_000, 100
    keys = oracle.gen_keys_uniform(n, G, 6)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 1e9, 1e-3, 6), 0.01, 0.0, 6)
    got, want = parity(ctx, keys, vals, G, "offset-1e9")
    rel = np.abs(got["m2"] - want["m2s"]) / want["m2s"]
    assert rel.max() < 1e-9


@pytest.mark.parametrize("G", [1, 2, 3, 31, 32, 33, 127, 128, 129, 255, 256, 257, 511, 512, 513, 777, 1023, 1024])
def test_group_counts_sweep(ctx, G):
    n = 123_457
    keys = oracle.gen_keys_uniform(n, G, G)
    vals = oracle.gen_values_normal(n, 5.0, 3.0, G)
    parity(ctx, keys, vals, G, f"G={G}")


@pytest.mark.parametrize("n", [0, 1, 2, 3, 4, 5, 2047, 2048, 2049, 4096 * 148 + 3, 2048 * 149])
def test_ragged_sizes(ctx, n):
    G = 17
    keys = oracle.gen_keys_uniform(n, G, n + 1)
    vals = oracle.gen_values_uniform(n, -3.0, 3.0, n + 1)
    parity(ctx, keys, vals, G, f"n={n}")


def test_empty_and_degenerate_groups(ctx):
    G = 8
    # group 0 empty, 1 all NaN, 2 only +inf, 3 +-inf, 4 single value, 5 constant, 6 zeros, 7 normal
    rows = [(1, np.nan), (1, np.nan), (2, np.inf), (3, np.inf), (3, -np.inf), (3, 2.0), (4, 42.0),
            (5, 7.0), (5, 7.0), (5, 7.0), (6, 0.0), (6, -0.0), (7, 1.5), (7, -2.5), (7, 0.25)]
    keys = np.array([r[0] for r in rows], np.int32)
    vals = np.array([r[1] for r in rows])
    got, _ = parity(ctx, keys, vals, G, "degenerate")
    assert got["count"][0] == 0 and math.isnan(got["mean"][0]) and got["min"][0] == np.inf
    assert got["max"][0] == -np.inf and got["sum"][0] == 0.0 and not math.copysign(1, got["sum"][0]) < 0
    assert got["count"][1] == 0
    assert got["count"][2] == 1 and got["sum"][2] == 0.0 and got["max"][2] == np.inf


def test_signed_zero_ties_follow_row_order(ctx):
    # a sequential `v < acc` scan keeps the first of equal values: +0 then -0 keeps +0
    n = 300_000
    G = 4
    keys = np.tile(np.arange(G, dtype=np.int32), n // G)
    vals = np.abs(oracle.gen_values_uniform(n, 0.5, 2.0, 9))  # positive
    vals[keys == 0] *= 1.0
    g0 = np.flatnonzero(keys == 0)
    vals[g0[1000]] = 0.0      # first zero of group 0: +0 -> min +0
    vals[g0[50000]] = -0.0
    g1 = np.flatnonzero(keys == 1)
    vals[g1[10]] = -0.0       # first zero of group 1: -0 -> min -0
    vals[g1[70000]] = 0.0
    g2 = np.flatnonzero(keys == 2)
    vals[g2] = -vals[g2]      # group 2 negative: max is its first zero
    vals[g2[123]] = -0.0
    vals[g2[60000]] = 0.0
    got, want = parity(ctx, keys, vals, G, "zeros")
    assert bits([got["min"][0]])[0] == bits([0.0])[0]
    assert bits([got["min"][1]])[0] == bits([-0.0])[0]
    assert bits([got["max"][2]])[0] == bits([-0.0])[0]


def test_heavy_skew_overflow_rounds(ctx):
    n, G = 200_000, 256
    keys = np.full(n, 7, np.int32)
    keys[::97] = 3
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 12)
    parity(ctx, keys, vals, G, "skew")


def test_out_of_range_key_raises(ctx):
    import winrapids_b200 as wb

    for bad in (5, -1):
        keys = np.array([0, 1, bad, 2], np.int32)
        vals = np.array([1.0, 2.0, 3.0, 4.0])
        with pytest.raises(wb.KeyOutOfRange):
            run_gpu(ctx, keys, vals, 3)
    # the context stays usable and the error is cleared
    parity(ctx, np.array([0, 1], np.int32), np.array([1.0, 2.0]), 2)


def test_nan_row_keys_are_not_checked(ctx):
    # rows masked out as NaN never index the accumulators (descriptive.rs:396-403, 606-620)
    keys = np.array([0, 9, 1], np.int32)
    vals = np.array([1.0, np.nan, 2.0])
    got = run_gpu(ctx, keys, vals, 2)
    assert list(got["count"]) == [1.0, 1.0]


def test_row_mask(ctx):
    n, G = 500_000, 64
    keys = oracle.gen_keys_uniform(n, G, 21)
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 21)
    a = oracle.gen_values_normal(n, 0.0, 1.0, 22)
    mask = oracle.filter_mask("gt", 0.0, a)
    got = run_gpu(ctx, keys, vals, G, mask=mask)
    want = oracle.moments_grouped_masked(vals, keys, mask, G)
    sel = np.unpackbits(mask.view(np.uint8), bitorder="little")[:n].astype(bool)
    check(got, want, abs_sums(keys, vals, G, sel), "mask")


@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("G", [128, 256, 512])
def test_compile_time_group_counts(ctx, G, masked):
    """128, 256 and 512 groups run their own kernel instantiations: zeros of both signs,
    +-inf, NaN, column overflow from a skewed key and a mask over many tiles all reach them."""
    n = 4096 * 300 + 77
    keys = oracle.gen_keys_uniform(n, G, 40 + G)
    keys[: 4096 * 3: 2] = 7  # one group overflows its column
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 40 + G)
    vals[::1009] = np.nan
    vals[3::7919] = np.inf
    vals[5::8191] = -np.inf
    vals[11::5003] = 0.0
    vals[13::6007] = -0.0
    if masked:
        a = oracle.gen_values_normal(n, 0.0, 1.0, 41 + G)
        a[4096 * 20: 4096 * 60] = -1.0  # whole tiles without a selected row
        mask = oracle.filter_mask("gt", -0.3, a)
        got = run_gpu(ctx, keys, vals, G, mask=mask)
        want = oracle.moments_grouped_masked(vals, keys, mask, G)
        sel = np.unpackbits(mask.view(np.uint8), bitorder="little")[:n].astype(bool)
        check(got, want, abs_sums(keys, vals, G, sel), f"G={G} masked")
    else:
        got = run_gpu(ctx, keys, vals, G)
        want = oracle.moments_grouped_mt(vals, keys, G, threads=8)
        check(got, want, abs_sums(keys, vals, G), f"G={G}")


def test_unaligned_inputs_take_the_plain_load_path(ctx):
    import torch

    n, G = 100_003, 50
    keys = oracle.gen_keys_uniform(n + 1, G, 31)
    vals = oracle.gen_values_normal(n + 1, 0.0, 1.0, 31)
    dk = torch.as_tensor(keys).cuda()[1:]
    dv = torch.as_tensor(vals).cuda()[1:]
    assert dk.data_ptr() % 16 != 0
    got = to_host(ctx.groupby_dense(dk, dv, G))
    want = oracle.moments_grouped_mt(vals[1:], keys[1:], G)
    check(got, want, abs_sums(keys[1:], vals[1:], G), "unaligned")


def test_sharded_states_merge_to_the_unsharded_result(ctx):
    import torch

    n, G = 1_500_000, 300
    keys = oracle.gen_keys_uniform(n, G, 41)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 100.0, 1.0, 41), 0.01, 0.001, 41)
    vals[::5000] = 0.0
    vals[1::7000] = -0.0
    dk, dv = torch.as_tensor(keys).cuda(), torch.as_tensor(vals).cuda()
    cuts = [0, 400_000, 400_000, 1_100_001, n]  # includes an empty shard
    states = []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        states.append(ctx.groupby_dense_state(dk[lo:hi], dv[lo:hi], G, row_offset=lo).clone())
    stacked = torch.cat(states)
    got = to_host(ctx.merge_states(stacked, len(states), G))
    ctx.sync()
    want = oracle.moments_grouped_mt(vals, keys, G)
    check(got, want, abs_sums(keys, vals, G), "sharded")


def test_run_to_run_stability(ctx):
    """count/min/max are bit-identical run to run; sum/mean/m2 agree within the contract
    tolerance (the in-tile summation order follows shared-memory atomic order)."""
    import torch

    n, G = 2_000_000, 256
    dk = torch.empty(n, dtype=torch.int32, device="cuda")
    dv = torch.empty(n, dtype=torch.float64, device="cuda")
    ctx.gen_keys_uniform(dk, G, 77)
    ctx.gen_values_uniform(dv, -1.0, 1.0, 77)
    a = to_host(ctx.groupby_dense(dk, dv, G))
    b = to_host(ctx.groupby_dense(dk, dv, G))
    for f in ("count", "min", "max"):
        assert np.array_equal(bits(a[f]), bits(b[f])), f
    absum = torch.zeros(G, dtype=torch.float64, device="cuda").index_add_(0, dk.long(), dv.abs()).cpu().numpy()
    assert np.all(np.abs(a["sum"] - b["sum"]) <= 1e-12 * absum)
    assert np.all(np.abs(a["m2"] - b["m2"]) <= 1e-9 * np.abs(a["m2"]))


def test_generators_match_the_host_recipe(ctx):
    import torch

    n = 100_001
    dk = torch.empty(n, dtype=torch.int32, device="cuda")
    du = torch.empty(n, dtype=torch.float64, device="cuda")
    dn = torch.empty(n, dtype=torch.float64, device="cuda")
    ctx.gen_keys_uniform(dk, 10_000, 5)
    ctx.gen_values_uniform(du, -1.0, 1.0, 5)
    ctx.gen_values_normal(dn, 1e9, 1e-3, 5)
    torch.cuda.synchronize()
    assert np.array_equal(dk.cpu().numpy(), oracle.gen_keys_uniform(n, 10_000, 5))
    assert np.array_equal(du.cpu().numpy(), oracle.gen_values_uniform(n, -1.0, 1.0, 5))
    hn = oracle.gen_values_normal(n, 1e9, 1e-3, 5)
    assert np.max(np.abs(dn.cpu().numpy() - hn)) <= 4 * np.spacing(1e9)
    v = dn.clone()
    ctx.gen_inject_nonfinite(v, 0.01, 0.001, 5)
    hv = oracle.inject_nonfinite(dn.cpu().numpy(), 0.01, 0.001, 5)
    gv = v.cpu().numpy()
    assert np.array_equal(np.isnan(gv), np.isnan(hv)) and np.array_equal(np.isinf(gv), np.isinf(hv))
    assert np.array_equal(gv[np.isinf(gv)], hv[np.isinf(hv)])


def test_descriptive_engine_mirror():
    import winrapids_b200 as wb

    eng = wb.DescriptiveEngine()
    st = eng.moments_grouped([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], [0, 0, 0, 1, 1, 1], 2)
    g0, g1 = st.group(0), st.group(1)
    assert g0.count == 3 and abs(g0.mean() - 2.0) < 1e-10 and abs(g0.variance(0) - 2 / 3) < 1e-10
    assert g1.count == 3 and abs(g1.mean() - 5.0) < 1e-10 and math.isnan(wb.MomentStats(1, 1, 1, 1, 0).variance(1))
    assert np.allclose(eng.mean_grouped([10.0, 20.0, 30.0, 40.0], [0, 1, 0, 1], 2), [20.0, 30.0])


@pytest.mark.slow
def test_config3_full_size_properties(ctx):
    """1e9 rows, 256 groups, U(-1,1): size-independent properties at the full configuration."""
    import torch

    n, G = 1_000_000_000, 256
    dk = torch.empty(n, dtype=torch.int32, device="cuda")
    dv = torch.empty(n, dtype=torch.float64, device="cuda")
    ctx.gen_keys_uniform(dk, G, 0)
    ctx.gen_values_uniform(dv, -1.0, 1.0, 0)
    a = to_host(ctx.groupby_dense(dk, dv, G))
    assert a["count"].sum() == n
    cnt = torch.bincount(dk, minlength=G).cpu().numpy()
    assert np.array_equal(a["count"], cnt.astype(np.float64))
    assert np.all(a["min"] >= -1.0) and np.all(a["max"] < 1.0)
    # a 4-way shard merge reproduces the unsharded result
    states, cuts = [], [0, 250_000_001, 500_000_000, 750_000_123, n]
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        states.append(ctx.groupby_dense_state(dk[lo:hi], dv[lo:hi], G, row_offset=lo).clone())
    b = to_host(ctx.merge_states(torch.cat(states), 4, G))
    ctx.sync()
    assert np.array_equal(a["count"], b["count"])
    assert np.array_equal(bits(a["min"]), bits(b["min"])) and np.array_equal(bits(a["max"]), bits(b["max"]))
    assert np.all(np.abs(a["sum"] - b["sum"]) <= 1e-12 * a["count"])
    assert np.all(np.abs(a["var_pop"] - 1.0 / 3.0) < 1e-3)
    # a sample of the rows checked directly against the oracle
    m = 4_000_000
    hk, hv = dk[:m].cpu().numpy(), dv[:m].cpu().numpy()
    c = to_host(ctx.groupby_dense(dk[:m], dv[:m], G))
    check(c, oracle.moments_grouped_mt(hv, hk, G), abs_sums(hk, hv, G), "C3 prefix")
