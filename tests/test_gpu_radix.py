"""The radix-partitioned int64-key groupby (count / sum / mean; table mode 'radix', the default for
many rows over a large key space) through the C ABI, against the oracle: plain f32 and f64
columns, mask + predicate + expression, edge keys and non-finite values, empty input, the
fallback to the global table when a bucket overflows its region (a heavy key, and crafted keys
whose hashes share their top 18 bits), and TABLE_FULL when the keys outnumber max_groups.  Every
call reports whether it fell back (tbgb_radix_fallback): the ordinary cases must not."""
import numpy as np
import pytest

import oracle
from parity import SUM_TOL, abs_sums

pytestmark = pytest.mark.gpu
SALT = 0x5EED5EED12345678
C1, C2 = 0xFF51AFD7ED558CCD, 0xC4CEB9FE1A85EC53


def dev(x):
    import torch

    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def fmix64_np(k):
    x = np.asarray(k).view(np.uint64).copy()
    with np.errstate(over="ignore"):
        x ^= x >> np.uint64(33)
        x *= np.uint64(C1)
        x ^= x >> np.uint64(33)
        x *= np.uint64(C2)
        x ^= x >> np.uint64(33)
    return x


def unfmix64_np(h):
    """Keys with chosen hashes: fmix64 is a bijection (xor-shifts by 33 undo themselves, odd
    multipliers have inverses mod 2^64)."""
    inv = lambda c: pow(c, -1, 1 << 64)  # noqa: E731
    x = np.asarray(h, dtype=np.uint64).copy()
    with np.errstate(over="ignore"):
        x ^= x >> np.uint64(33)
        x *= np.uint64(inv(C2))
        x ^= x >> np.uint64(33)
        x *= np.uint64(inv(C1))
        x ^= x >> np.uint64(33)
    return x.view(np.int64)


def run(ctx, keys, a, max_groups, fallback=0, **kw):
    """The radix groupby; `fallback`: the fallback bits the call must report (0: the radix passes
    produced the result themselves)."""
    import winrapids_b200 as wb

    ctx.set_table_mode("radix")
    try:
        gk, out = ctx.groupby_hash(dev(keys), dev(a) if not hasattr(a, "cuda") else a, max_groups,
                                   fields=wb.SUMCOUNT_FIELDS, **kw)
        bits = ctx.radix_fallback()
    finally:
        ctx.set_table_mode("auto")
    assert bits == fallback, f"fallback bits {bits}, expected {fallback}"
    return gk.cpu().numpy(), {f: t.cpu().numpy() for f, t in out.items()}


def compare(gk, got, keys, v, live, label):
    want = oracle.groupby_i64(keys[live], v[live])
    order = np.argsort(gk, kind="stable")
    assert np.array_equal(gk[order], want["keys"]), f"{label} keys ({gk.size} vs {want['keys'].size})"
    got = {f: x[order] for f, x in got.items()}
    c = want["counts"]
    assert np.array_equal(got["count"], c), f"{label} count"
    codes = np.searchsorted(want["keys"], keys[live])
    absum = abs_sums(codes, v[live], want["keys"].size)
    assert np.all(np.abs(got["sum"] - want["sums"]) <= SUM_TOL * absum), f"{label} sum"
    cnt = np.where(c > 0, c, 1.0)
    ok = np.where(c > 0, np.abs(got["mean"] - want["sums"] / cnt) <= SUM_TOL * absum / cnt, np.isnan(got["mean"]))
    assert np.all(ok), f"{label} mean"


def test_f32_values_plain(ctx):
    n, ids = 6_000_011, 1 << 21
    keys = oracle.gen_keys_ids(n, ids, SALT, 3)
    vals = oracle.gen_values_lognormal_f32(n, 0.0, 1.0, 3)
    gk, got = run(ctx, keys, vals, ids)
    compare(gk, got, keys, vals.astype(np.float64), np.ones(n, bool), "f32")


def test_f32_values_across_the_fixed_point_range(ctx):
    """f32 sums are exact 64-bit fixed point for magnitudes in [2^-13, 2^E) and f64 atomics
    outside it: groups that mix tiny, huge, negative, zero, subnormal and non-finite values, with
    a group's positive and negative values cancelling, take both parts and their sum."""
    rng = np.random.default_rng(11)
    n, ids = 4_000_003, 1 << 20
    keys = oracle.gen_keys_ids(n, ids, SALT, 5)
    mag = np.float32(2.0) ** rng.integers(-40, 40, n).astype(np.float32)
    vals = (rng.uniform(1.0, 2.0, n).astype(np.float32) * mag).astype(np.float32)
    vals[rng.random(n) < 0.5] *= np.float32(-1.0)
    vals[rng.random(n) < 0.01] = np.float32(0.0)
    vals[rng.random(n) < 0.01] = np.float32(1e-42)  # subnormal
    vals[rng.random(n) < 0.01] = np.float32(3e38)
    vals[rng.random(n) < 0.01] = np.float32(np.nan)
    vals[rng.random(n) < 0.005] = np.float32(np.inf)
    edge = np.float32(2.0) ** np.float32(-13)
    vals[rng.random(n) < 0.01] = edge  # the smallest magnitude on the fixed-point side
    vals[rng.random(n) < 0.01] = np.nextafter(edge, np.float32(0.0))  # the largest below it
    gk, got = run(ctx, keys, vals, ids)
    compare(gk, got, keys, vals.astype(np.float64), np.ones(n, bool), "f32 range")


def test_f64_values_plain_with_nonfinite_and_edge_keys(ctx):
    rng = np.random.default_rng(7)
    n = 3_000_000
    keys = rng.integers(-2**62, 2**62, n).astype(np.int64)
    pool = np.array([np.iinfo(np.int64).min, np.iinfo(np.int64).max, 0, -1, 1], dtype=np.int64)
    pick = rng.random(n) < 1e-4  # about 60 rows of each edge key: present, but no heavy hitter
    keys[pick] = pool[rng.integers(0, pool.size, pick.sum())]
    vals = rng.normal(size=n)
    vals[rng.random(n) < 0.02] = np.nan
    vals[rng.random(n) < 0.01] = np.inf
    vals[rng.random(n) < 0.01] = -np.inf
    vals[keys == -1] = np.nan  # a key whose rows are all NaN: a group with count 0
    gk, got = run(ctx, keys, vals, 4_000_000)
    compare(gk, got, keys, vals, np.ones(n, bool), "f64 edge")
    assert got["count"][gk == -1][0] == 0.0 and np.isnan(got["mean"][gk == -1][0])


@pytest.mark.parametrize("dtype", ["f64", "f32"])
def test_mask_predicate_expression(ctx, dtype):
    n, ids = 4_000_003, 1 << 20
    keys = oracle.gen_keys_ids(n, ids, SALT, 5)
    a = oracle.gen_values_normal(n, 0.0, 1.0, 6)
    b = oracle.gen_values_normal(n, 1.0, 1.0, 7)
    c = oracle.gen_values_normal(n, 0.0, 2.0, 8)
    if dtype == "f32":
        a, b, c = (x.astype(np.float32) for x in (a, b, c))
    rng = np.random.default_rng(9)
    live_mask = rng.random(n) < 0.7
    words = np.zeros((n + 63) // 64, dtype=np.uint64)
    idx = np.nonzero(live_mask)[0]
    np.bitwise_or.at(words, idx // 64, np.left_shift(np.uint64(1), (idx % 64).astype(np.uint64)))
    kw = dict(b=dev(b), c=dev(c), expr="a*b+c", pred=">", threshold=-0.5, mask=dev(words.view(np.int64)))
    gk, got = run(ctx, keys, a, ids, **kw)
    a64, b64, c64 = (np.asarray(x, np.float64) for x in (a, b, c))
    v = oracle.map2("a + b", oracle.map2("a * b", a64, b64), c64)
    live = live_mask & (a64 > -0.5)
    compare(gk, got, keys, v, live, f"masked {dtype}")
    # the predicate alone on an f32 column keeps 12-byte rows (no expression)
    gk, got = run(ctx, keys, a, ids, pred=">", threshold=0.25)
    compare(gk, got, keys, a64, a64 > 0.25, f"pred {dtype}")


def test_empty_input(ctx):
    gk, got = run(ctx, np.zeros(0, np.int64), np.zeros(0, np.float64), 1 << 20)
    assert gk.size == 0


def test_heavy_key_overflows_a_first_pass_bucket(ctx):
    """60 % of the rows on one key: its first-pass bucket outgrows its region and the global table
    recomputes the whole result."""
    n, ids = 3_000_000, 1 << 20
    keys = oracle.gen_keys_ids(n, ids, SALT, 11)
    keys[np.random.default_rng(1).random(n) < 0.6] = 424242
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 11)
    gk, got = run(ctx, keys, vals, ids, fallback=1)
    compare(gk, got, keys, vals, np.ones(n, bool), "heavy key")


def test_crafted_hashes_overflow_a_final_bucket(ctx):
    """1,500 distinct keys (two rows each) whose hashes share their top 18 bits, among ordinary keys:
    their first-pass bucket still fits its region, their final bucket does not (second pass); the
    global table recomputes the result."""
    rng = np.random.default_rng(12)
    n_ord = 2_000_000
    ordinary = oracle.gen_keys_ids(n_ord, 1 << 20, SALT, 12)
    low = rng.choice(1 << 40, 1500, replace=False).astype(np.uint64)
    crafted = unfmix64_np((np.uint64(0x2ABCD) << np.uint64(46)) | low)
    assert np.all((fmix64_np(crafted) >> np.uint64(46)) == 0x2ABCD)
    keys = np.concatenate([ordinary, crafted, crafted])
    vals = rng.normal(size=keys.size)
    gk, got = run(ctx, keys, vals, 1 << 21, fallback=1)
    compare(gk, got, keys, vals, np.ones(keys.size, bool), "crafted")


def test_more_keys_than_max_groups_is_table_full(ctx):
    import winrapids_b200 as wb

    n = 1_000_000
    keys = oracle.gen_keys_ids(n, 1 << 20, SALT, 13)
    vals = np.ones(n)
    with pytest.raises(wb.TableFull):
        run(ctx, keys, vals, 100_000)
