"""m3 / m4 in the same pass (the m3s / m4s of moments_grouped, descriptive.rs:421-432) on every
path -- the column kernel, the global table (dense and int64 keys), sharded states -- against
the oracle's exact sums.  Tolerance: |got - want| <= 1e-9 * sum |v - r|^k over the group's
finite values (m3 can be near zero, so the scale is the absolute sum, not m3 itself)."""
import numpy as np
import pytest

import oracle
from parity import abs_sums, check, to_host

pytestmark = pytest.mark.gpu
TOL = 1e-9


def dev(x):
    import torch

    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def abs_pow(keys, vals, mean, k, G, live=None):
    v = np.asarray(vals, np.float64)
    ok = np.isfinite(v) if live is None else (np.isfinite(v) & live)
    kk = np.asarray(keys)[ok]
    return np.bincount(kk, weights=np.abs(v[ok] - mean[kk]) ** k, minlength=G)


def check_m34(got, want, keys, vals, G, label, live=None):
    c = want["counts"]
    r = np.where(c > 0, want["sums"] / np.where(c > 0, c, 1.0), 0.0)
    for f, w, k in (("m3", want["m3s"], 3), ("m4", want["m4s"], 4)):
        scale = abs_pow(keys, vals, r, k, G, live)
        err = np.abs(got[f] - w)
        assert np.all(err <= TOL * scale), f"{label} {f}: worst {np.max(err / np.maximum(scale, 1e-300))}"


FIELDS = ("count", "sum", "min", "max", "mean", "m2", "var_pop", "var_samp", "m3", "m4")


@pytest.mark.parametrize("G,mu,sigma", [(256, 0.0, 1.0), (7, 5.0, 2.0), (1000, 1e9, 1e-3)])
def test_column_kernel(ctx, G, mu, sigma):
    n = 1_500_000
    keys = oracle.gen_keys_uniform(n, G, 3)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, mu, sigma, 3), 0.01, 0.002, 3)
    got = to_host(ctx.groupby_dense(dev(keys), dev(vals), G, out=ctx.alloc_moments(G, FIELDS)))
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8, m34=True)
    check(got, want, abs_sums(keys, vals, G), f"G={G}")
    check_m34(got, want, keys, vals, G, f"G={G}")


def test_column_kernel_default_skips_higher_moments(ctx):
    """Without m3 / m4 outputs the same call computes the other fields identically."""
    n, G = 500_000, 256
    keys = oracle.gen_keys_uniform(n, G, 4)
    vals = oracle.gen_values_uniform(n, -1.0, 1.0, 4)
    a = to_host(ctx.groupby_dense(dev(keys), dev(vals), G))
    b = to_host(ctx.groupby_dense(dev(keys), dev(vals), G, out=ctx.alloc_moments(G, FIELDS)))
    for f in ("count", "min", "max"):
        assert np.array_equal(a[f], b[f])


@pytest.mark.parametrize("mode", ["local", "direct", "range", "sweep"])
def test_table_dense(ctx, mode):
    n, G = 1_000_000, 5000
    keys = oracle.gen_keys_uniform(n, G, 5)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 1e9, 1e-3, 5), 0.01, 0.001, 5)
    ctx.set_table_mode(mode)
    try:
        got = to_host(ctx.groupby_dense(dev(keys), dev(vals), G, out=ctx.alloc_moments(G, FIELDS)))
    finally:
        ctx.set_table_mode("auto")
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8, m34=True)
    check(got, want, abs_sums(keys, vals, G), mode)
    check_m34(got, want, keys, vals, G, mode)


@pytest.mark.parametrize("mode", ["local", "direct"])
def test_table_hash(ctx, mode):
    n, ids = 1_000_000, 50_000
    keys = oracle.gen_keys_ids(n, ids, 0x77, 6)
    vals = oracle.gen_values_normal(n, 2.0, 3.0, 6) ** 3
    ctx.set_table_mode(mode)
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(vals), ids, fields=FIELDS)
    finally:
        ctx.set_table_mode("auto")
    got = to_host(out)
    order = np.argsort(gk.cpu().numpy())
    got = {f: a[order] for f, a in got.items()}
    want = oracle.groupby_i64(keys, vals, m34=True)
    assert np.array_equal(gk.cpu().numpy()[order], want["keys"])
    codes = np.searchsorted(want["keys"], keys)
    check(got, want, abs_sums(codes, vals, want["keys"].size), f"hash {mode}")
    check_m34(got, want, codes, vals, want["keys"].size, f"hash {mode}")


@pytest.mark.parametrize("G", [256, 3000])
def test_sharded_states(ctx, G):
    import torch

    n, P = 900_000, 3
    keys = oracle.gen_keys_uniform(n, G, 7)
    vals = oracle.gen_values_normal(n, 10.0, 4.0, 7)
    sb = ctx.state_bytes(G) // 8
    states = torch.empty(P * sb, dtype=torch.float64, device="cuda")
    bounds = np.linspace(0, n, P + 1).astype(np.int64)
    for r in range(P):
        lo, hi = bounds[r], bounds[r + 1]
        ctx.groupby_dense_state(dev(keys[lo:hi]), dev(vals[lo:hi]), G, row_offset=int(lo), state=states[r * sb:])
    got = to_host(ctx.merge_states(states, P, G, out=ctx.alloc_moments(G, FIELDS)))
    ctx.sync()
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8, m34=True)
    check(got, want, abs_sums(keys, vals, G), "states")
    check_m34(got, want, keys, vals, G, "states")


def test_descriptive_engine_returns_m3_m4():
    import winrapids_b200 as wb

    n, G = 200_000, 50
    keys = oracle.gen_keys_uniform(n, G, 8)
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 8) ** 2
    g = wb.DescriptiveEngine(0).moments_grouped(vals, keys, G)
    want = oracle.moments_grouped(vals, keys, G, m34=True)
    assert np.array_equal(g.counts, want["counts"])
    got = {"m3": g.m3s, "m4": g.m4s}
    check_m34(got, want, keys, vals, G, "engine")
    s = g.group(3)
    assert s.skewness(True) > 0  # chi-square-like values are right-skewed


NO_EXTREMA = ("count", "sum", "mean", "m2", "var_pop", "var_samp", "m3", "m4")


@pytest.mark.parametrize("mode", ["local", "auto"])
def test_table_hash_without_extrema(ctx, mode):
    """Outputs without min / max: the int64-key shared-table path that queues rows per warp and
    leaves the extrema arrays out, with m3 / m4."""
    n, ids = 1_000_000, 50_000
    keys = oracle.gen_keys_ids(n, ids, 0x78, 7)
    vals = oracle.gen_values_normal(n, 2.0, 3.0, 7) ** 3
    ctx.set_table_mode(mode)
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(vals), ids, fields=NO_EXTREMA)
    finally:
        ctx.set_table_mode("auto")
    assert "min" not in out and "max" not in out
    got = to_host(out)
    order = np.argsort(gk.cpu().numpy())
    got = {f: a[order] for f, a in got.items()}
    want = oracle.groupby_i64(keys, vals, m34=True)
    assert np.array_equal(gk.cpu().numpy()[order], want["keys"])
    codes = np.searchsorted(want["keys"], keys)
    # count / sum / mean / m2 / variances as `check` has them, extrema taken from the oracle
    got["min"], got["max"] = want["mins"], want["maxs"]
    check(got, want, abs_sums(codes, vals, want["keys"].size), f"hash no-extrema {mode}")
    check_m34(got, want, codes, vals, want["keys"].size, f"hash no-extrema {mode}")
