"""GPU parity of the global-table groupby (dense keys beyond 1024 groups, int64 hash keys,
fused filter + expression, f32 columns) through the C ABI, against the oracle."""
import numpy as np
import pytest

import oracle
from parity import SUM_TOL, abs_sums, bits, check, to_host

pytestmark = pytest.mark.gpu

SALT = 0x5EED5EED12345678
MODES = ("local", "direct", "bucket", "range", "sweep")


def dev(x):
    import torch

    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def dev_mask(m):
    return None if m is None else dev(np.ascontiguousarray(m, dtype=np.uint64).view(np.int64))


def host_value(a, b=None, c=None, expr="a"):
    """The oracle's value column: map2 compositions of the reference (two roundings for a*b+c)."""
    a64 = np.asarray(a, dtype=np.float64)
    b64 = None if b is None else np.asarray(b, dtype=np.float64)
    c64 = None if c is None else np.asarray(c, dtype=np.float64)
    if expr == "a":
        return a64
    if expr == "a*b+c":
        return oracle.map2("a + b", oracle.map2("a * b", a64, b64), c64)
    return oracle.map2({"a+b": "a + b", "a-b": "a - b", "a*b": "a * b", "a*b+1": "a * b + 1.0"}[expr], a64, b64)


def host_mask(n, a=None, pred=None, thr=0.0, mask=None):
    words = (n + 63) // 64
    m = np.full(words, ~np.uint64(0), dtype=np.uint64) if mask is None else np.asarray(mask, np.uint64).copy()
    if pred is not None:
        m &= oracle.filter_mask({">": "gt", ">=": "ge", "<": "lt", "<=": "le", "not_nan": "not_nan",
                                 "finite": "finite"}[pred], thr, np.asarray(a, dtype=np.float64))
    if n % 64:
        m[-1] &= np.uint64((1 << (n % 64)) - 1)
    return m


def rows_of(mask, n):
    return ((mask[np.arange(n) // 64] >> (np.arange(n) % 64).astype(np.uint64)) & np.uint64(1)).astype(bool)


# ---- dense keys through the table ----------------------------------------------------

@pytest.mark.parametrize("mode", MODES + ("auto",))
def test_stress_shape_10000_groups(ctx, mode):
    """Numerical-stress shape: int32 keys in [0,10000), 1e9 + N(0,1e-3), 1% NaN, 0.1% +-inf."""
    n, G, seed = 2_000_000, 10_000, 5
    keys = oracle.gen_keys_uniform(n, G, seed)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 1e9, 1e-3, seed), 0.01, 0.001, seed)
    ctx.set_table_mode(mode)
    try:
        got = to_host(ctx.groupby_dense(dev(keys), dev(vals), G))
    finally:
        ctx.set_table_mode("auto")
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8)
    check(got, want, abs_sums(keys, vals, G), f"stress {mode}")


@pytest.mark.parametrize("G", [1025, 4096, 65536])
def test_dense_many_groups(ctx, G):
    n, seed = 1_500_000, 11
    keys = oracle.gen_keys_uniform(n, G, seed)
    vals = oracle.gen_values_normal(n, 0.0, 1.0, seed)
    got = to_host(ctx.groupby_dense(dev(keys), dev(vals), G))
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8)
    check(got, want, abs_sums(keys, vals, G), f"G={G}")


def test_dense_table_empty_input(ctx):
    import torch

    G = 3000
    got = to_host(ctx.groupby_dense(torch.empty(0, dtype=torch.int32, device="cuda"),
                                    torch.empty(0, dtype=torch.float64, device="cuda"), G))
    assert np.all(got["count"] == 0) and np.all(got["sum"] == 0) and not np.any(np.signbit(got["sum"]))
    assert np.all(got["min"] == np.inf) and np.all(got["max"] == -np.inf)
    assert np.all(np.isnan(got["mean"])) and np.all(np.isnan(got["var_pop"])) and np.all(got["m2"] == 0)


def test_dense_table_key_out_of_range(ctx):
    import winrapids_b200 as wb

    n, G = 100_000, 2000
    keys = oracle.gen_keys_uniform(n, G, 3)
    keys[777] = G
    with pytest.raises(wb.KeyOutOfRange):
        ctx.groupby_dense(dev(keys), dev(np.ones(n)), G)
    ctx.groupby_dense(dev(keys[:700]), dev(np.ones(700)), G)  # the context stays usable


@pytest.mark.parametrize("mode,G", [(m, 1500) for m in MODES] + [("auto", 5000), ("range", 12000)])
def test_dense_table_zero_ties_and_infs(ctx, mode, G):
    """+-0 ties resolve to the first zero in row order; +-inf rows count, leave the sum (5,000 and
    12,000 groups: group ranges whose shift and first-zero code live in the global slots)."""
    rng = np.random.default_rng(7)
    n = 400_000
    keys = rng.integers(0, G, n).astype(np.int32)
    vals = np.where(rng.random(n) < 0.5, 0.0, -0.0)
    vals[rng.random(n) < 0.01] = np.inf
    vals[rng.random(n) < 0.01] = -np.inf
    vals[rng.random(n) < 0.02] = np.nan
    pos = rng.random(n) < 0.3
    vals[pos] = np.abs(vals[pos])  # more +0 than -0, in random order
    ctx.set_table_mode(mode)
    try:
        got = to_host(ctx.groupby_dense(dev(keys), dev(vals), G))
    finally:
        ctx.set_table_mode("auto")
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8)
    check(got, want, abs_sums(keys, vals, G), f"zeros {mode}")


def test_dense_state_merge_many_groups(ctx):
    """Row shards of a 3000-group table: per-shard states, merged in shard order."""
    import torch

    n, G, seed, P = 900_000, 3000, 21, 3
    keys = oracle.gen_keys_uniform(n, G, seed)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 5.0, 2.0, seed), 0.01, 0.002, seed)
    vals[::9973] = -0.0
    vals[5::9967] = 0.0
    sb = ctx.state_bytes(G) // 8
    states = torch.empty(P * sb, dtype=torch.float64, device="cuda")
    bounds = np.linspace(0, n, P + 1).astype(np.int64)
    for r in range(P):
        lo, hi = bounds[r], bounds[r + 1]
        ctx.groupby_dense_state(dev(keys[lo:hi]), dev(vals[lo:hi]), G, row_offset=int(lo), state=states[r * sb:])
    got = to_host(ctx.merge_states(states, P, G))
    ctx.sync()
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8)
    check(got, want, abs_sums(keys, vals, G), "sharded table")


@pytest.mark.parametrize("G", [1500, 9000, 30000])
@pytest.mark.parametrize("f32", [False, True])
def test_dense_range_ragged_unaligned(ctx, G, f32):
    """Group ranges in shared memory: a row count that is not a multiple of four, columns that
    start on and off a 16-byte boundary, a row mask, a predicate and a*b+c (1, 3 and 8 ranges)."""
    import torch

    n, seed = 1_000_003, 51
    keys = oracle.gen_keys_uniform(n + 1, G, seed)
    cols = [oracle.gen_values_normal(n + 1, 0.0, 1.0, seed + i) for i in (1, 2, 3)]
    if f32:
        cols = [x.astype(np.float32) for x in cols]
    cols[0][::777] = np.nan
    cols[0][3::1201] = np.inf
    user = host_mask(n)
    user[::5] = np.uint64(0x0F0F0F0F0F0F0F0F)
    dk = torch.as_tensor(keys).cuda()
    dc = [torch.as_tensor(x).cuda() for x in cols]
    ctx.set_table_mode("range")
    try:
        for off in (0, 1):
            a, b, c = (x[off:off + n] for x in dc)
            got = to_host(ctx.groupby_dense_columns(dk[off:off + n], a, G, b=b, c=c, expr="a*b+c", pred=">",
                                                    threshold=-0.5, mask=dev_mask(user)))
            ha, hb, hc = (x[off:off + n].astype(np.float64) for x in cols)
            m = host_mask(n, ha, ">", -0.5, user)
            v = host_value(ha, hb, hc, "a*b+c")
            k = keys[off:off + n]
            want = oracle.moments_grouped_mt(v, k, G, threads=8, mask=m)
            check(got, want, abs_sums(k, v, G, rows_of(m, n)), f"range G={G} f32={f32} off={off}")
    finally:
        ctx.set_table_mode("auto")


@pytest.mark.parametrize("G", [1500, 9000])
@pytest.mark.parametrize("f32", [False, True])
def test_dense_sweep_ragged_masked(ctx, G, f32):
    """Rank and sweep (mode 6): a row count that is not a multiple of four, a row mask, a predicate,
    NaN / +-inf / +-0 values, keys 16-byte aligned (offsets 0 and 4) and not (offset 1: the call
    takes the group-range kernel instead); one range at 1,500 groups, three at 9,000."""
    import torch

    n, seed = 1_000_003, 53
    keys = oracle.gen_keys_uniform(n + 4, G, seed)
    a = oracle.gen_values_normal(n + 4, 0.0, 1.0, seed + 1)
    a[::777] = np.nan
    a[3::1201] = np.inf
    a[5::1301] = -np.inf
    a[7::901] = 0.0
    a[9::1103] = -0.0
    if f32:
        a = a.astype(np.float32)
    user = host_mask(n)
    user[::5] = np.uint64(0x0F0F0F0F0F0F0F0F)
    dk = torch.as_tensor(keys).cuda()
    da = torch.as_tensor(a).cuda()
    ctx.set_table_mode("sweep")
    try:
        for off in (0, 1, 4):
            got = to_host(ctx.groupby_dense_columns(dk[off:off + n], da[off:off + n], G, pred=">=", threshold=-1.0,
                                                    mask=dev_mask(user)))
            ha = a[off:off + n].astype(np.float64)
            m = host_mask(n, ha, ">=", -1.0, user)
            k = keys[off:off + n]
            want = oracle.moments_grouped_mt(ha, k, G, threads=8, mask=m)
            check(got, want, abs_sums(k, ha, G, rows_of(m, n)), f"sweep G={G} f32={f32} off={off}")
    finally:
        ctx.set_table_mode("auto")


@pytest.mark.parametrize("mode", ["range", "sweep"])
def test_dense_range_key_out_of_range_only_when_selected(ctx, mode):
    """Keys outside [0, G) raise only on rows that the mask and the predicate select."""
    import winrapids_b200 as wb

    n, G = 200_001, 9000
    keys = oracle.gen_keys_uniform(n, G, 8)
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 8)
    keys[100], keys[70_001], keys[n - 1] = G + 5, -3, G
    vals[70_001] = -1.0
    user = host_mask(n)
    for r in (100, n - 1):
        user[r // 64] &= ~np.uint64(1 << (r % 64))
    ctx.set_table_mode(mode)
    try:
        got = to_host(ctx.groupby_dense_columns(dev(keys), dev(vals), G, pred=">", threshold=0.0,
                                                mask=dev_mask(user)))
        with pytest.raises(wb.KeyOutOfRange):
            ctx.groupby_dense(dev(keys), dev(vals), G)
        again = to_host(ctx.groupby_dense_columns(dev(keys), dev(vals), G, pred=">", threshold=0.0,
                                                  mask=dev_mask(user)))
    finally:
        ctx.set_table_mode("auto")
    m = host_mask(n, vals, ">", 0.0, user)
    k = np.where((keys >= 0) & (keys < G), keys, 0).astype(np.int32)
    want = oracle.moments_grouped_mt(vals, k, G, threads=8, mask=m)
    check(got, want, abs_sums(k, vals, G, rows_of(m, n)), f"{mode} oor masked")
    for f in ("count", "min", "max"):
        assert np.array_equal(bits(got[f]), bits(again[f])), f


# ---- fused filter + expression over dense keys ------------------------------------------

@pytest.mark.parametrize("G", [256, 5000])
@pytest.mark.parametrize("expr", ["a", "a+b", "a-b", "a*b", "a*b+1", "a*b+c"])
def test_dense_columns_filter_expr(ctx, G, expr):
    n, seed = 700_000, 31
    keys = oracle.gen_keys_uniform(n, G, seed)
    a = oracle.gen_values_normal(n, 0.0, 1.0, seed + 1)
    b = oracle.gen_values_normal(n, 0.0, 1.0, seed + 2)
    c = oracle.gen_values_normal(n, 0.0, 1.0, seed + 3)
    a[::1001] = np.nan
    user = host_mask(n)
    user[::3] = np.uint64(0xF0F0F0F0F0F0F0F0)
    got = to_host(ctx.groupby_dense_columns(dev(keys), dev(a), G, b=dev(b), c=dev(c), expr=expr, pred=">",
                                            threshold=0.0, mask=dev_mask(user)))
    m = host_mask(n, a, ">", 0.0, user)
    v = host_value(a, b, c, expr)
    want = oracle.moments_grouped_mt(v, keys, G, threads=8, mask=m)
    check(got, want, abs_sums(keys, v, G, rows_of(m, n)), f"{expr} G={G}")


@pytest.mark.parametrize("pred,thr", [(">=", 0.5), ("<", -0.25), ("<=", 0.0), ("not_nan", 0.0), ("finite", 0.0)])
def test_dense_columns_predicates_f32(ctx, pred, thr):
    n, G, seed = 300_000, 700, 41
    keys = oracle.gen_keys_uniform(n, G, seed)
    a = oracle.gen_values_normal(n, 0.0, 1.0, seed).astype(np.float32)
    a[::997] = np.nan
    a[1::991] = np.inf
    a[2::983] = -np.inf
    got = to_host(ctx.groupby_dense_columns(dev(keys), dev(a), G, pred=pred, threshold=thr))
    a64 = a.astype(np.float64)
    m = host_mask(n, a64, pred, thr)
    want = oracle.moments_grouped_mt(a64, keys, G, threads=8, mask=m)
    check(got, want, abs_sums(keys, a64, G, rows_of(m, n)), f"f32 {pred}")


# ---- int64 keys through the hash table ----------------------------------------------------

def hash_check(gk, got, want, v, keys, m, label, fields=None):
    """Sort the GPU groups by key and compare with the oracle's key-sorted groups."""
    order = np.argsort(gk, kind="stable")
    gk = gk[order]
    got = {f: a[order] for f, a in got.items()}
    assert np.array_equal(gk, want["keys"]), f"{label} group keys"
    live = rows_of(m, keys.size) if m is not None else np.ones(keys.size, bool)
    codes = np.searchsorted(want["keys"], keys[live])
    absum = abs_sums(codes, v[live], want["keys"].size)
    if fields is None:
        check(got, want, absum, label)
        return
    c = want["counts"]
    assert np.array_equal(got["count"], c), f"{label} count"
    assert np.all(np.abs(got["sum"] - want["sums"]) <= SUM_TOL * absum), f"{label} sum"
    d = oracle.derived(want)
    cnt = np.where(c > 0, c, 1.0)
    ok = np.where(c > 0, np.abs(got["mean"] - d["mean"]) <= SUM_TOL * absum / cnt, np.isnan(got["mean"]))
    assert np.all(ok), f"{label} mean"


@pytest.mark.parametrize("mode", MODES)
def test_fused_pipeline_shape(ctx, mode):
    """Fused pipeline shape: int64 Zipf(1.1) keys over 1,000,000 ids, filter a>0, v=a*b+c (scaled rows)."""
    import winrapids_b200 as wb

    n, seed, ids = 3_000_000, 2, 1_000_000
    cdf = oracle.zipf_cdf(ids, 1.1)
    keys = oracle.gen_keys_cdf(n, cdf, SALT, seed)
    a = oracle.gen_values_normal(n, 0.0, 1.0, seed + 1)
    b = oracle.gen_values_normal(n, 0.0, 1.0, seed + 2)
    c = oracle.gen_values_normal(n, 0.0, 1.0, seed + 3)
    ctx.set_table_mode(mode)
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(a), ids, b=dev(b), c=dev(c), expr="a*b+c", pred=">",
                                   threshold=0.0)
    finally:
        ctx.set_table_mode("auto")
    got = to_host(out)
    gk = gk.cpu().numpy()
    m = host_mask(n, a, ">", 0.0)
    v = host_value(a, b, c, "a*b+c")
    want = oracle.groupby_i64(keys, v, mask=m)
    hash_check(gk, got, want, v, keys, m, f"pipeline {mode}")


@pytest.mark.parametrize("mode", MODES)
def test_high_cardinality_shape(ctx, mode):
    """High-cardinality shape: int64 keys uniform over random ids, f32 LogNormal(0,1), sum/count/mean."""
    import winrapids_b200 as wb

    n, seed, ids = 4_000_000, 4, 1 << 20
    keys = oracle.gen_keys_ids(n, ids, SALT, seed)
    vals = oracle.gen_values_lognormal_f32(n, 0.0, 1.0, seed)
    ctx.set_table_mode(mode)
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(vals), ids, fields=wb.SUMCOUNT_FIELDS)
    finally:
        ctx.set_table_mode("auto")
    got = to_host(out)
    v64 = vals.astype(np.float64)
    want = oracle.groupby_i64(keys, v64)
    hash_check(gk.cpu().numpy(), got, want, v64, keys, None, f"highcard {mode}", fields=wb.SUMCOUNT_FIELDS)


@pytest.mark.parametrize("mode", MODES)
def test_hash_edge_keys_and_values(ctx, mode):
    """INT64_MIN / INT64_MAX / 0 / -1 keys, NaN-only groups, +-0 ties, +-inf, rows masked out."""
    rng = np.random.default_rng(99)
    n = 200_000
    pool = np.array([np.iinfo(np.int64).min, np.iinfo(np.int64).max, 0, -1, 1, 12345], dtype=np.int64)
    keys = np.where(rng.random(n) < 0.5, pool[rng.integers(0, pool.size, n)], rng.integers(-2**62, 2**62, n))
    keys = keys.astype(np.int64)
    vals = rng.normal(size=n)
    vals[rng.random(n) < 0.05] = 0.0
    vals[rng.random(n) < 0.05] = -0.0
    vals[rng.random(n) < 0.01] = np.inf
    vals[rng.random(n) < 0.01] = -np.inf
    vals[keys == 12345] = np.nan  # a group with NaN rows only
    user = host_mask(n)
    user[::5] = np.uint64(0)
    ctx.set_table_mode(mode)
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(vals), n, mask=dev_mask(user))
    finally:
        ctx.set_table_mode("auto")
    got = to_host(out)
    want = oracle.groupby_i64(keys, vals, mask=user)
    assert 12345 in want["keys"] and np.iinfo(np.int64).min in want["keys"]
    hash_check(gk.cpu().numpy(), got, want, vals, keys, user, f"edge {mode}")


PIPELINE_FIELDS = ("count", "sum", "mean", "m2", "var_pop", "var_samp")


def check_no_extrema(got, want, absum, label):
    got = dict(got)
    got["min"], got["max"] = want["mins"], want["maxs"]
    check(got, want, absum, label)


@pytest.mark.parametrize("mode", ["auto", "local"])
def test_fused_pipeline_bench_fields(ctx, mode):
    """The fused pipeline with the bench's outputs (no extrema): the int64-key shared table with
    rows queued per warp, Zipf head keys and a long tail through the global table."""
    n, seed, ids = 3_000_000, 5, 1_000_000
    cdf = oracle.zipf_cdf(ids, 1.1)
    keys = oracle.gen_keys_cdf(n, cdf, SALT, seed)
    a = oracle.gen_values_normal(n, 0.0, 1.0, seed + 1)
    b = oracle.gen_values_normal(n, 0.0, 1.0, seed + 2)
    c = oracle.gen_values_normal(n, 0.0, 1.0, seed + 3)
    ctx.set_table_mode(mode)
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(a), ids, b=dev(b), c=dev(c), expr="a*b+c", pred=">",
                                   threshold=0.0, fields=PIPELINE_FIELDS)
    finally:
        ctx.set_table_mode("auto")
    got = to_host(out)
    gk = gk.cpu().numpy()
    m = host_mask(n, a, ">", 0.0)
    v = host_value(a, b, c, "a*b+c")
    want = oracle.groupby_i64(keys, v, mask=m)
    order = np.argsort(gk, kind="stable")
    assert np.array_equal(gk[order], want["keys"])
    live = rows_of(m, n)
    codes = np.searchsorted(want["keys"], keys[live])
    check_no_extrema({f: x[order] for f, x in got.items()}, want, abs_sums(codes, v[live], want["keys"].size),
                     f"pipeline fields {mode}")


def test_hash_edge_keys_without_extrema(ctx):
    """INT64_MIN / INT64_MAX / 0 / -1 keys, a NaN-only group, +-inf and masked rows, without extrema
    (the queued shared-table path, INT64_MIN through the global table's sentinel slot)."""
    rng = np.random.default_rng(98)
    n = 400_000
    pool = np.array([np.iinfo(np.int64).min, np.iinfo(np.int64).max, 0, -1, 1, 12345], dtype=np.int64)
    keys = np.where(rng.random(n) < 0.5, pool[rng.integers(0, pool.size, n)], rng.integers(-2**62, 2**62, n))
    keys = keys.astype(np.int64)
    vals = rng.normal(size=n)
    vals[rng.random(n) < 0.01] = np.inf
    vals[rng.random(n) < 0.01] = -np.inf
    vals[keys == 12345] = np.nan
    user = host_mask(n)
    user[::7] = np.uint64(0)
    ctx.set_table_mode("local")
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(vals), n, mask=dev_mask(user), fields=PIPELINE_FIELDS)
    finally:
        ctx.set_table_mode("auto")
    got = to_host(out)
    gk = gk.cpu().numpy()
    want = oracle.groupby_i64(keys, vals, mask=user)
    assert 12345 in want["keys"] and np.iinfo(np.int64).min in want["keys"]
    order = np.argsort(gk, kind="stable")
    assert np.array_equal(gk[order], want["keys"])
    live = rows_of(user, n)
    codes = np.searchsorted(want["keys"], keys[live])
    check_no_extrema({f: x[order] for f, x in got.items()}, want, abs_sums(codes, vals[live], want["keys"].size),
                     "edge no-extrema")


def test_hash_filter_rejects_everything(ctx):
    n = 50_000
    keys = np.arange(n, dtype=np.int64)
    a = -np.abs(np.random.default_rng(1).normal(size=n)) - 1.0
    gk, out = ctx.groupby_hash(dev(keys), dev(a), 1000, pred=">", threshold=0.0)
    assert gk.numel() == 0 and out["count"].numel() == 0


def test_hash_table_full(ctx):
    import winrapids_b200 as wb

    n = 100_000
    keys = np.arange(n, dtype=np.int64) * 7919
    with pytest.raises(wb.TableFull):
        ctx.groupby_hash(dev(keys), dev(np.ones(n)), 5000)
    gk, out = ctx.groupby_hash(dev(keys[:100]), dev(np.ones(100)), 5000)  # usable afterwards
    assert gk.numel() == 100


def test_hash_empty_input(ctx):
    import torch

    gk, out = ctx.groupby_hash(torch.empty(0, dtype=torch.int64, device="cuda"),
                               torch.empty(0, dtype=torch.float64, device="cuda"), 10)
    assert gk.numel() == 0


# ---- generators of the new key / value columns ---------------------------------------------

def test_generators_match_numpy(ctx):
    import torch

    n, first = 1_000_003, 123_456
    cdf = oracle.zipf_cdf(100_000, 1.1)
    k = torch.empty(n, dtype=torch.int64, device="cuda")
    ctx.gen_keys_cdf(k, dev(cdf), SALT, 9, first_row=first)
    assert np.array_equal(k.cpu().numpy(), oracle.gen_keys_cdf(n, cdf, SALT, 9, start=first))
    ctx.gen_keys_ids(k, 1 << 28, SALT, 9, first_row=first)
    assert np.array_equal(k.cpu().numpy(), oracle.gen_keys_ids(n, 1 << 28, SALT, 9, start=first))
    f = torch.empty(n, dtype=torch.float32, device="cuda")
    ctx.gen_values_lognormal_f32(f, 0.0, 1.0, 9, first_row=first)
    host = oracle.gen_values_lognormal_f32(n, 0.0, 1.0, 9, start=first)
    got = f.cpu().numpy()
    # exp / log / cos of CUDA and of the host libm may differ in the last f64 bit, which can
    # move the f32 rounding by one ulp at most
    ulp = np.abs(got.view(np.int32).astype(np.int64) - host.view(np.int32).astype(np.int64))
    assert ulp.max() <= 1 and np.mean(ulp) < 1e-3
