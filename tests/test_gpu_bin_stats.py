"""GPU parity of the bin statistics (tbgb_fused_bin_stats) against the reference's own kernels
(src/winrapids/kernels/bin_stats.cu, compiled from the reference tree into
oracle/_ref/libref_bin_stats.so and run on the same device arrays) and against the oracle's
serial restatement.

Tolerances: count, min, max, first and last are bit-exact; sum and sum_sq are within
1e-12 * sum(|v|) and 1e-12 * sum(v*v) of the serial loop (the product sums in parallel), with
the same NaN / +-inf outcome; mean, variance and std follow from them."""
import ctypes as C
import math
from pathlib import Path

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_bin_stats.so"


def dev(x):
    import torch

    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def ref_stats(data, bounds):
    """The reference kernel on the device (None when the reference build is absent)."""
    if not REF_LIB.exists():
        return None
    import torch

    L = C.CDLL(str(REF_LIB))
    d = np.atleast_2d(np.asarray(data, np.float64))
    ncol, n = d.shape
    nb = len(bounds) - 1
    D, B = dev(d.reshape(-1)), dev(np.asarray(bounds, np.int64))
    outs = {k: torch.empty(ncol * max(nb, 1), dtype=torch.float64, device="cuda")
            for k in ("sum", "sum_sq", "min", "max", "first", "last")}
    cnt = torch.empty(max(nb, 1), dtype=torch.int32, device="cuda")
    args = [C.c_void_p(D.data_ptr()), C.c_void_p(B.data_ptr())] + [C.c_void_p(outs[k].data_ptr()) for k in
                                                                   ("sum", "sum_sq", "min", "max", "first", "last")]
    args += [C.c_void_p(cnt.data_ptr()), C.c_int(nb)]
    if ncol == 1:
        rc = L.ref_fused_bin_stats(*args, None)
    else:
        rc = L.ref_fused_bin_stats_multi(*args, C.c_int(ncol), C.c_longlong(n), None)
    assert rc == 0
    torch.cuda.synchronize()
    res = {k: host(v)[:ncol * nb].reshape(ncol, nb) for k, v in outs.items()}
    res["count"] = host(cnt)[:nb]
    return res


def bits(a):
    return np.ascontiguousarray(a, np.float64).view(np.uint64)


def close_sum(got, want, mag):
    got, want = np.asarray(got), np.asarray(want)
    fin = np.isfinite(want)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[~fin & ~np.isnan(want)], want[~fin & ~np.isnan(want)])
    assert np.all(np.abs(got[fin] - want[fin]) <= 1e-12 * mag[fin] + 1e-300)


def magnitudes(d, bounds):
    d = np.asarray(d, np.float64)
    a, q = [], []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        seg = d[lo:hi]
        seg = seg[np.isfinite(seg)]
        a.append(np.sum(np.abs(seg)))
        q.append(np.sum(seg * seg))
    return np.array(a), np.array(q)


def check(got, want, d, bounds, col=None):
    """got: product outputs of one column; want: reference/oracle outputs of that column."""
    mag, magq = magnitudes(d, bounds)
    assert np.array_equal(got["count"], want["count"])
    for f in ("min", "max", "first", "last"):
        g, w = got[f], want[f]
        assert np.array_equal(np.isnan(g), np.isnan(w)), f
        assert np.array_equal(bits(g)[~np.isnan(w)], bits(w)[~np.isnan(w)]), f
    close_sum(got["sum"], want["sum"], mag)
    close_sum(got["sum_sq"], want["sum_sq"], magq)
    c = want["count"].astype(np.float64)
    with np.errstate(invalid="ignore", divide="ignore"):
        mean = np.where(c > 0, want["sum"] / np.where(c > 0, c, 1.0), np.nan)
    close_sum(got["mean"], mean, mag / np.where(c > 0, c, 1.0))
    var = got["variance"]
    assert np.array_equal(np.isnan(var), np.isnan(oracle_var(want)))
    assert np.all(var[~np.isnan(var)] >= 0.0)
    assert np.allclose(got["std"], np.sqrt(var), equal_nan=True, rtol=0, atol=0)


def oracle_var(w):
    c = w["count"].astype(np.float64)
    with np.errstate(invalid="ignore", divide="ignore"):
        m = w["sum"] / np.where(c > 0, c, 1.0)
        v = np.where(c > 1, w["sum_sq"] / np.where(c > 0, c, 1.0) - m * m, np.nan)
    return np.where(v < 0, 0.0, v)


def values(rng, n, nonfinite=True):
    v = rng.standard_normal(n) * 100.0 + 3.0
    if nonfinite and n:
        r = rng.random(n)
        v[r < 0.01] = np.nan
        v[(r >= 0.01) & (r < 0.015)] = np.inf
        v[(r >= 0.015) & (r < 0.02)] = -np.inf
        v[(r >= 0.02) & (r < 0.03)] = 0.0
        v[(r >= 0.03) & (r < 0.04)] = -0.0
    return v


def bounds_from_sizes(sizes, start=0):
    return np.concatenate([[start], start + np.cumsum(sizes)]).astype(np.int64)


LAYOUTS = {
    "uniform_416": lambda rng, n: bounds_from_sizes(np.full(n // 416, 416)),
    "random_sizes": lambda rng, n: bounds_from_sizes(rng.integers(0, 3000, size=n // 1500)),
    "tiny_and_empty": lambda rng, n: bounds_from_sizes(rng.integers(0, 4, size=n // 2)),
    "mixed_giant": lambda rng, n: bounds_from_sizes(
        np.concatenate([rng.integers(0, 20, 500), [n // 2], rng.integers(1, 5000, 60)])),
    "one_bin": lambda rng, n: np.array([0, n], np.int64),
    "partial_cover": lambda rng, n: bounds_from_sizes(rng.integers(1, 9000, size=40), start=777),
}


def test_reference_kernel_build_present():
    """The comparisons against the reference's own kernel need oracle/_ref (built by
    __graft_entry__.build() where the reference tree exists)."""
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libref_bin_stats.so not built: only the oracle restatement is compared")


@pytest.mark.parametrize("layout", list(LAYOUTS))
def test_bin_stats_vs_reference_and_oracle(ctx, layout):
    rng = np.random.default_rng(len(layout))
    n = 400_000
    d = values(rng, n)
    bnd = LAYOUTS[layout](rng, n)
    bnd = bnd[bnd <= n] if bnd[-1] > n else bnd
    got = {k: host(v) for k, v in ctx.fused_bin_stats(dev(d), dev(bnd)).items()}
    want = oracle.bin_stats(d, bnd)
    check(got, want, d, bnd)
    ref = ref_stats(d, bnd)
    if ref is not None:
        r = {k: (v if k == "count" else v[0]) for k, v in ref.items()}
        check(got, r, d, bnd)
        # the oracle restatement itself against the reference kernel
        assert np.array_equal(ref["count"], want["count"])
        for f in ("min", "max", "first", "last"):
            assert np.array_equal(bits(r[f])[~np.isnan(r[f])], bits(want[f])[~np.isnan(want[f])]), f


def test_bin_stats_multi_column(ctx):
    import winrapids_b200 as wb

    rng = np.random.default_rng(9)
    n = 250_003
    cols = {"price": values(rng, n), "size": values(rng, n, nonfinite=False), "notional": values(rng, n)}
    bnd = bounds_from_sizes(rng.integers(0, 700, size=n // 350))
    bnd = bnd[bnd <= n]
    got = wb.fused_multi_column_bin_stats({k: dev(v) for k, v in cols.items()}, dev(bnd))
    stacked = np.stack(list(cols.values()))
    ref = ref_stats(stacked, bnd)
    for j, (name, d) in enumerate(cols.items()):
        g = {k: host(v) for k, v in got[name].items()}
        check(g, oracle.bin_stats(d, bnd), d, bnd)
        if ref is not None:
            check(g, {k: (v if k == "count" else v[j]) for k, v in ref.items()}, d, bnd)


def test_bin_stats_python_wrapper_and_edges(ctx):
    import torch

    import winrapids_b200 as wb

    r = wb.fused_bin_stats([1.0, 2.0, 3.0, math.nan, 5.0, -0.0, 0.0, 7.0], [0, 3, 3, 5, 8])
    assert set(r) == {"count", "sum", "sum_sq", "min", "max", "first", "last", "mean", "variance", "std"}
    assert list(host(r["count"])) == [3, 0, 2, 3]
    assert host(r["sum"])[0] == 6.0 and math.isnan(host(r["sum"])[1]) and math.isnan(host(r["min"])[2])
    mn = host(r["min"])[3]
    assert mn == 0.0 and math.copysign(1.0, mn) == -1.0   # first of the zeros, as the serial scan keeps
    assert host(r["last"])[2] == 5.0
    assert abs(host(r["variance"])[0] - 2.0 / 3.0) < 1e-15
    # no ticks: every bin empty
    e = ctx.fused_bin_stats(torch.zeros(0, dtype=torch.float64, device="cuda"), dev(np.zeros(4, np.int64)))
    assert list(host(e["count"])) == [0, 0, 0] and np.all(np.isnan(host(e["sum"])))
    # no bins
    z = ctx.fused_bin_stats(dev(np.ones(10)), dev(np.zeros(1, np.int64)))
    assert host(z["count"]).size == 0


@pytest.mark.parametrize("bnd", [[0, 10, 5, 20], [0, 5, 205], [-3, 4], [0, 100, 100, 400]])
def test_bin_stats_invalid_boundaries_are_reported(ctx, bnd):
    import winrapids_b200 as wb

    d = dev(np.arange(200, dtype=np.float64))
    with pytest.raises(wb.InvalidArgument):
        ctx.fused_bin_stats(d, dev(np.asarray(bnd, np.int64)))
    ok = ctx.fused_bin_stats(d, dev(np.asarray([0, 50, 200], np.int64)))  # the context stays usable
    assert list(host(ok["count"])) == [50, 150]
