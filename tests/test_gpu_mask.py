"""GPU parity of the mask-not-filter plumbing against the oracle's restatements:
predicate masks (FilterJit::filter_mask), mask algebra (MaskOp / mask_*), per-tile
TileColumnStats, tile-skip masks, tile skipping inside a groupby, and the Frame /
GroupByBuilder caller surface.

Tolerances: masks, popcounts, skip flags, tile counts and tile min / max are bit-exact;
a tile's finite sum is within 1e-12 * sum(|x|) of the serial Kahan sum (it is
computed as a compensated parallel sum), and its non-finite cases (NaN, a trailing
infinity) are exact."""
import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from parity import abs_sums, check, to_host

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "reference_vectors.json").read_text())["cases"]
ORC_PRED = {">": "gt", ">=": "ge", "<": "lt", "<=": "le", "not_nan": "not_nan", "finite": "finite"}


def dev(x):
    import torch

    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def words_dev(m):
    return dev(np.ascontiguousarray(m, dtype=np.uint64).view(np.int64))


def words_host(t):
    return t.cpu().numpy().view(np.uint64)


def hexwords(xs):
    return np.array([int(x, 16) for x in xs], dtype=np.uint64)


def column(rng, n, kind="mixed"):
    v = rng.standard_normal(n)
    if kind == "mixed" and n:
        r = rng.random(n)
        v[r < 0.02] = np.nan
        v[(r >= 0.02) & (r < 0.03)] = np.inf
        v[(r >= 0.03) & (r < 0.04)] = -np.inf
        v[(r >= 0.04) & (r < 0.06)] = 0.0
        v[(r >= 0.06) & (r < 0.08)] = -0.0
    return v


def random_mask(rng, n, density=0.5):
    bits = rng.random(n) < density
    m = np.zeros((n + 63) // 64, np.uint64)
    for w in range(m.size):
        seg = bits[w * 64:(w + 1) * 64]
        m[w] = np.uint64(int("".join("1" if b else "0" for b in seg[::-1]) or "0", 2))
    return m


def rows_of(mask, n):
    idx = np.arange(n)
    return ((mask[idx // 64] >> (idx % 64).astype(np.uint64)) & np.uint64(1)).astype(bool)


# ---- predicate masks ----

@pytest.mark.parametrize("n", [0, 1, 63, 64, 65, 2047, 2048, 2049, 100_003])
@pytest.mark.parametrize("pred", [">", ">=", "<", "<=", "not_nan", "finite"])
def test_filter_mask_vs_oracle(ctx, n, pred):
    rng = np.random.default_rng(n * 7 + len(pred))
    v = column(rng, n)
    thr = 0.25
    got = words_host(ctx.filter_mask(dev(v), pred, thr)) if n else np.zeros(0, np.uint64)
    want = oracle.filter_mask(ORC_PRED[pred], thr, v)
    assert np.array_equal(got, want)


def test_filter_mask_none_and_f32(ctx):
    rng = np.random.default_rng(5)
    n = 10_001
    v32 = column(rng, n).astype(np.float32)
    got = words_host(ctx.filter_mask(dev(v32), ">", -0.5))
    assert np.array_equal(got, oracle.filter_mask("gt", -0.5, v32.astype(np.float64)))
    allrows = words_host(ctx.filter_mask(dev(v32), "none"))
    assert np.array_equal(rows_of(allrows, n), np.ones(n, bool))
    assert allrows[-1] >> np.uint64(n % 64) == 0  # trailing bits zero


@pytest.mark.parametrize("n", [1, 130, 4097, 300_001])
def test_filter_mask_with_input_mask(ctx, n):
    rng = np.random.default_rng(n)
    v = column(rng, n)
    inm = random_mask(rng, n, 0.3)
    got = words_host(ctx.filter_mask(dev(v), "<", 0.1, in_mask=words_dev(inm)))
    want = oracle.mask_and(oracle.filter_mask("lt", 0.1, v), inm)
    assert np.array_equal(got, want)
    # in place (the output aliases the input mask)
    t = words_dev(inm)
    ctx.filter_mask(dev(v), "<", 0.1, in_mask=t, out=t)
    assert np.array_equal(words_host(t), want)


@pytest.mark.parametrize("case", [c for c in GOLDEN if c["kind"] == "filter_mask"], ids=lambda c: c["cite"])
def test_filter_jit_golden(case):
    import winrapids_b200 as wb

    vals = [float.fromhex(v) if v not in ("nan", "inf", "-inf") else float(v) for v in case["values"]]
    thr = float.fromhex(case["threshold"])
    jit = wb.FilterJit()
    m = jit.filter_mask(f"v > {thr!r}", vals)
    assert m.size == (len(vals) + 63) // 64
    assert np.array_equal(m & hexwords(case["check"]), hexwords(case["expect"]))


def test_filter_jit_cache_and_constants():
    import winrapids_b200 as wb
    from winrapids_b200.frame import PRED_FINITE, PRED_NOT_NAN

    jit = wb.FilterJit()
    jit.filter_mask("v > 1.5", [1.0, 2.0, 3.0])
    jit.filter_mask("v > 1.5", [1.0, 2.0, 3.0])
    assert len(jit.cache) == 1  # filter_jit.rs:630-637 filter_cached
    v = [1.0, math.nan, math.inf, -2.0]
    assert jit.filter_mask(PRED_NOT_NAN, v)[0] == 0b1101
    assert jit.filter_mask(PRED_FINITE, v)[0] == 0b1001


# ---- mask algebra ----

@pytest.mark.parametrize("n_rows", [1, 64, 65, 1000, 262_145])
def test_mask_algebra_vs_oracle(ctx, n_rows):
    rng = np.random.default_rng(n_rows)
    a, b = random_mask(rng, n_rows, 0.4), random_mask(rng, n_rows, 0.6)
    A, B = words_dev(a), words_dev(b)
    assert np.array_equal(words_host(ctx.mask_and(A, B)), oracle.mask_and(a, b))
    assert np.array_equal(words_host(ctx.mask_or(A, B)), oracle.mask_or(a, b))
    assert np.array_equal(words_host(ctx.mask_xor(A, B)), oracle.mask_xor(a, b))
    assert np.array_equal(words_host(ctx.mask_not(A, n_rows)), oracle.mask_not(a, n_rows))
    assert ctx.mask_popcount(A, n_rows) == oracle.mask_popcount(a, n_rows)
    # garbage in the trailing bits is not counted
    g = a.copy()
    g[-1] |= ~np.uint64(0) << np.uint64(n_rows % 64) if n_rows % 64 else np.uint64(0)
    assert ctx.mask_popcount(words_dev(g), n_rows) == oracle.mask_popcount(a, n_rows)
    # in place
    ctx.mask_and(A, B, out=A)
    assert np.array_equal(words_host(A), oracle.mask_and(a, b))


@pytest.mark.parametrize("case", [c for c in GOLDEN if c["kind"].startswith("mask_")], ids=lambda c: c["cite"])
def test_mask_op_golden(case):
    import winrapids_b200 as wb

    op = wb.MaskOp()
    k = case["kind"]
    if k == "mask_binary":
        f = {"and": op.mask_and, "or": op.mask_or, "xor": op.mask_xor}[case["op"]]
        assert np.array_equal(f(hexwords(case["a"]), hexwords(case["b"])), hexwords(case["expect"]))
    elif k == "mask_not":
        assert np.array_equal(op.mask_not(hexwords(case["a"]), case["n_rows"]), hexwords(case["expect"]))
    elif k == "mask_popcount":
        m = hexwords(case["mask"])
        assert op.mask_popcount_gpu(words_dev(m), m.size, case["n_rows"]) == case["expect"]
    else:  # mask_and_popcount
        a, b = words_dev(hexwords(case["a"])), words_dev(hexwords(case["b"]))
        both = op.mask_and_gpu(a, b, 2)
        assert op.mask_popcount_gpu(both, 2, case["n_rows"]) == case["expect"]


def test_mask_errors(ctx):
    import winrapids_b200 as wb

    a = words_dev(np.zeros(2, np.uint64))
    with pytest.raises(wb.InvalidArgument):
        ctx.mask_not(a, 200)          # needs ceil(200 / 64) = 4 words
    assert ctx.mask_popcount(a, 10) == 0   # words past ceil(n_rows / 64) are ignored
    with pytest.raises(wb.InvalidArgument):
        ctx.mask_popcount(a, 129)     # needs 3 words
    with pytest.raises(wb.InvalidArgument):
        ctx.mask_and(a, words_dev(np.zeros(3, np.uint64)))
    with pytest.raises(wb.EntryNotFound):
        ctx.tile_skip_mask(ctx.tile_stats(dev(np.ones(8)), 4), "not_nan", 0.0)


# ---- tile statistics ----

def check_tiles(got, want, vals, tile_rows):
    from winrapids_b200.frame import tile_stats_numpy

    g = tile_stats_numpy(got)
    assert g.size == want.size
    assert np.array_equal(g["count"], want["count"]) and np.array_equal(g["n_valid"], want["n_valid"])
    assert np.array_equal(g["reserved"], np.zeros(g.size, np.uint64))
    assert np.array_equal(g["min"].view(np.uint64), want["min"].view(np.uint64)), "min bits"
    assert np.array_equal(g["max"].view(np.uint64), want["max"].view(np.uint64)), "max bits"
    v = np.asarray(vals, np.float64)
    for t in range(g.size):
        seg = v[t * tile_rows:(t + 1) * tile_rows]
        ws, gs = float(want["sum"][t]), float(g["sum"][t])
        if not math.isfinite(ws):
            assert (math.isnan(gs) and math.isnan(ws)) or gs == ws, (t, gs, ws)
        else:
            assert abs(gs - ws) <= 1e-12 * float(np.sum(np.abs(seg))) + 1e-300, (t, gs, ws)


@pytest.mark.parametrize("tile_rows", [1, 7, 64, 1000, 65536])
@pytest.mark.parametrize("kind", ["clean", "mixed"])
def test_tile_stats_vs_oracle(ctx, tile_rows, kind):
    rng = np.random.default_rng(tile_rows)
    n = 200_003
    v = column(rng, n, kind) * 1e3
    got = ctx.tile_stats(dev(v), tile_rows)
    check_tiles(got, oracle.tile_stats(v, tile_rows), v, tile_rows)


def test_tile_stats_edge_cases(ctx):
    inf, nan = math.inf, math.nan
    v = np.array([1.0, 2.0, inf, 3.0, 1.0, 2.0, 3.0, -inf, 7.0, nan, -0.0, 0.0, nan, nan, nan, nan,
                  0.0, -0.0, 0.0, -0.0])
    got = ctx.tile_stats(dev(v), 4)
    check_tiles(got, oracle.tile_stats(v, 4), v, 4)
    v32 = np.array([3.5, -1.25, 8.0], np.float32)
    check_tiles(ctx.tile_stats(dev(v32), 2), oracle.tile_stats(v32.astype(np.float64), 2), v32, 2)


@pytest.mark.parametrize("case", [c for c in GOLDEN if c["kind"] == "tile_stats_global"], ids=lambda c: c["cite"])
def test_tile_global_golden(ctx, case):
    from winrapids_b200 import frame as fr

    vals = ([float(i) for i in range(case["arange"])] if "arange" in case
            else [float.fromhex(x) for x in case["values"]])
    st = ctx.tile_stats(dev(np.array(vals)), case["tile_rows"])
    e = case["expect"]
    assert st.shape[0] == case["n_tiles"]
    assert fr.global_min(st) == float.fromhex(e["min"]) and fr.global_max(st) == float.fromhex(e["max"])
    assert fr.global_count(st) == e["count"]
    assert abs(fr.global_mean(st) - float.fromhex(e["mean"])) < case["tol"]


@pytest.mark.parametrize("pred", [">", ">=", "<", "<="])
def test_tile_skip_vs_oracle(ctx, pred):
    rng = np.random.default_rng(3)
    n, tr = 100_000, 1000
    v = np.cumsum(rng.standard_normal(n))  # a random walk: tiles have narrow ranges
    st_dev = ctx.tile_stats(dev(v), tr)
    st = oracle.tile_stats(v, tr)
    for thr in (float(np.median(v)), float(v.min()) - 1, float(v.max()) + 1, math.nan):
        got = ctx.tile_skip_mask(st_dev, pred, thr).cpu().numpy()
        assert np.array_equal(got, oracle.tile_skip(st, ORC_PRED[pred], thr)), thr


@pytest.mark.parametrize("tile_rows", [1, 5, 64, 100, 65536])
def test_mask_skip_tiles(ctx, tile_rows):
    rng = np.random.default_rng(tile_rows)
    n = 70_001
    n_tiles = (n + tile_rows - 1) // tile_rows
    skip = (rng.random(n_tiles) < 0.5).astype(np.uint8)
    inm = random_mask(rng, n, 0.7)
    keep = ~skip.astype(bool)[np.arange(n) // tile_rows]
    for m in (None, inm):
        got = words_host(ctx.mask_skip_tiles(dev(skip), tile_rows, n, mask=None if m is None else words_dev(m)))
        want_rows = keep & (rows_of(m, n) if m is not None else True)
        assert np.array_equal(rows_of(got, n), want_rows)
        if n % 64:
            assert got[-1] >> np.uint64(n % 64) == 0


def test_tile_skip_filter_equals_full_filter(ctx):
    """Skipping tiles ruled out by their statistics changes no mask bit."""
    rng = np.random.default_rng(11)
    n, tr = 1_000_003, 4096
    v = np.cumsum(rng.standard_normal(n)) * 0.01 + np.linspace(0, 100, n)
    thr = 90.0
    V = dev(v)
    skip = ctx.tile_skip_mask(ctx.tile_stats(V, tr), ">", thr)
    assert int(skip.sum().item()) > 0.8 * skip.numel()
    base = ctx.mask_skip_tiles(skip, tr, n)
    got = words_host(ctx.filter_mask(V, ">", thr, in_mask=base))
    assert np.array_equal(got, oracle.filter_mask("gt", thr, v))


@pytest.mark.parametrize("hash_keys", [False, True])
def test_groupby_with_tile_skip_mask(ctx, hash_keys):
    """The table path reads no column of a masked-out row and agrees with the oracle."""
    rng = np.random.default_rng(21)
    n, tr, G = 500_000, 8192, 3000
    a = np.linspace(-1, 1, n) + rng.standard_normal(n) * 1e-3
    keys = rng.integers(0, G, n).astype(np.int32)
    thr = 0.6
    A = dev(a)
    skip = ctx.tile_skip_mask(ctx.tile_stats(A, tr), ">", thr)
    m = ctx.mask_skip_tiles(skip, tr, n)
    rows = rows_of(words_host(m), n) & (a > thr)
    if hash_keys:
        k64 = keys.astype(np.int64) * 1_000_003 - 7
        gk, out = ctx.groupby_hash(dev(k64), A, 2 * G, pred=">", threshold=thr, mask=m)
        order = np.argsort(gk.cpu().numpy())
        got = {f: t.cpu().numpy()[order] for f, t in out.items()}
        want = oracle.groupby_i64(k64, a, mask=oracle.filter_mask("gt", thr, a))
        wk = want["keys"]
        assert np.array_equal(np.sort(gk.cpu().numpy()), wk)
        check(got, want, abs_sums(np.searchsorted(wk, k64[rows]), a[rows], wk.size), "hash+skip")
    else:
        out = ctx.groupby_dense_columns(dev(keys), A, G, pred=">", threshold=thr, mask=m)
        want = oracle.moments_grouped_masked(a, keys, oracle.filter_mask("gt", thr, a), G)
        check(to_host(out), want, abs_sums(keys, a, G, rows), "dense+skip")


# ---- Frame / GroupByBuilder ----

def test_frame_groupby(ctx):
    import winrapids_b200 as wb

    df = wb.from_columns({"ticker_id": [0, 0, 1, 1, 2], "close": [149.0, 150.1, 20.0, 22.0, 7.5]})
    assert df.n_rows == 5 and len(df) == 5 and df.columns == ["ticker_id", "close"]
    assert repr(df) == "Frame(n_rows=5, columns=['ticker_id', 'close'])"
    gb = df.groupby("ticker_id")
    assert repr(gb) == "GroupByBuilder(key='ticker_id', n_groups=3)"
    s = gb.sum("close")
    assert np.allclose(s.sums, [299.1, 42.0, 7.5], rtol=0, atol=1e-12)
    st = gb.stats("close")
    assert np.array_equal(st.counts, [2.0, 2.0, 1.0])
    assert np.allclose(st.means(), [149.55, 21.0, 7.5])
    v = st.variances()
    assert np.allclose(v[:2], [np.var([149.0, 150.1], ddof=1), 2.0]) and np.isnan(v[2])
    assert st.n_active() == 3 and repr(st) == "GroupByResult(n_groups=3, n_active=3)"
    with pytest.raises(KeyError):
        df.groupby("nope")
    with pytest.raises(TypeError):
        df.groupby("close")
    with pytest.raises(TypeError):
        gb.stats("ticker_id")
    with pytest.raises(ValueError):
        wb.from_columns({"a": [1, 2], "b": [1.0]})


def test_frame_filter_is_mask_not_filter(ctx):
    import winrapids_b200 as wb

    rng = np.random.default_rng(8)
    n, G = 300_001, 50
    keys = rng.integers(0, G, n).astype(np.int32)
    price = np.linspace(100, 300, n) + rng.standard_normal(n)
    df = wb.from_columns({"k": keys, "price": price})
    df.tile_rows = 4096
    hot = df.filter("price", "v > 240.0")
    assert hot.n_rows == n and not df.is_filtered() and hot.is_filtered()
    sel = price > 240.0
    assert hot.active_rows() == int(sel.sum())
    r = hot.groupby("k").stats("price")
    want = oracle.moments_grouped_masked(price, keys, oracle.filter_mask("gt", 240.0, price), G)
    assert np.array_equal(r.counts, want["counts"])
    absum = abs_sums(keys, price, G, sel)
    assert np.all(np.abs(r.sums - want["sums"]) <= 1e-12 * absum)
    # a second filter ANDs into the mask
    both = hot.filter("price", "v <= 260.0")
    assert both.active_rows() == int((sel & (price <= 260.0)).sum())
    assert hot.active_rows() == int(sel.sum())  # the parent frame's mask is unchanged
    gi = df.group_index_for("k", G - 1)
    assert gi is df.group_index_for("k", G - 1)


@pytest.mark.parametrize("G", [1, 256, 1000])
def test_dense_predicate_route_with_zero_tiles(ctx, G):
    """A predicate on a plain f64 column with <= 1024 groups runs as a row mask plus the masked
    column kernel, which skips tiles whose mask words are all zero; results as the oracle's, and
    counts / extrema bit-identical to the table path's."""
    rng = np.random.default_rng(G)
    n = 3_000_017
    a = column(rng, n) * 10.0
    keys = rng.integers(0, G, n).astype(np.int32)
    # rows outside [0.3n, 0.35n) and [0.8n, 0.81n) masked out: most 2048-row tiles are all zero
    inm_rows = np.zeros(n, bool)
    inm_rows[int(0.3 * n):int(0.35 * n)] = True
    inm_rows[int(0.8 * n):int(0.81 * n)] = True
    inm = np.packbits(inm_rows, bitorder="little")
    inm = np.concatenate([inm, np.zeros((-inm.size) % 8, np.uint8)]).view(np.uint64)
    fields = ("count", "sum", "min", "max", "mean", "m2", "var_pop", "var_samp", "m3", "m4")
    for mask in (None, inm):
        M = None if mask is None else words_dev(mask)
        out = ctx.groupby_dense_columns(dev(keys), dev(a), G, pred=">=", threshold=-2.5, mask=M,
                                        out=ctx.alloc_moments(G, fields))
        fm = oracle.filter_mask("ge", -2.5, a)
        if mask is not None:
            fm = oracle.mask_and(fm, mask)
        want = oracle.moments_grouped_masked(a, keys, fm, G, m34=True)
        rows = rows_of(fm, n)
        got = to_host(out)
        check(got, want, abs_sums(keys, a, G, rows), f"G={G} masked={mask is not None}")
        ctx.set_table_mode("direct")
        try:
            t = to_host(ctx.groupby_dense_columns(dev(keys), dev(a), G, pred=">=", threshold=-2.5, mask=M))
        finally:
            ctx.set_table_mode("auto")
        for f in ("count", "min", "max"):
            assert np.array_equal(got[f].view(np.uint64), t[f].view(np.uint64)), f
