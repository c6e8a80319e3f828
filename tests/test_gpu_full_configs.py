"""Parity at the full sizes of the groupby configurations, against the oracle (the reference's
CPU path restated, exact Kulisch sums), through the C ABI:

  low-cardinality   10^9 rows, int32 keys in [0,256), f64 U(-1,1), all six aggregates
  numerical stress  2*10^8 rows, int32 keys in [0,10000), 1e9 + N(0,1e-3), 1% NaN, 0.1% +-inf
  fused pipeline    10^8 rows, int64 Zipf(1.1) keys over 10^6 ids, filter a > 0, v = a*b + c
  high cardinality  2.5*10^8 rows over 2^28 random int64 ids (f32 LogNormal), sum/count/mean:
                    the 2^28-group table with its real key space (about 1.7*10^8 groups)

Inputs are generated on the device by the counter-based generators and copied to the host, so
the oracle sees exactly the bytes the kernels read.  Tolerances as in tests/parity.py.  The
int64-key oracle runs over key-disjoint buckets on all host cores; the buckets are formed by a
device-side permutation of the rows, which cannot change an exact (order-independent) sum."""
import os
import threading

import numpy as np
import pytest

import oracle
from parity import SUM_TOL, check, to_host

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
SALT = 0x5EED5EED12345678


def threads():
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except Exception:
        return os.cpu_count() or 1


def need_host_gb(gb):
    try:
        import psutil

        if psutil.virtual_memory().available < gb * (1 << 30):
            pytest.skip(f"needs about {gb} GB of free host memory")
    except ImportError:
        pass


def dense_absum(dk, dv, G):
    """sum |v| over each group's finite values, on the device (the tolerance scale)."""
    import torch

    fin = torch.isfinite(dv)
    w = torch.where(fin, dv.abs(), torch.zeros((), dtype=torch.float64, device=dv.device))
    out = torch.zeros(G, dtype=torch.float64, device=dv.device)
    step = 1 << 27
    for lo in range(0, dv.numel(), step):
        out.index_add_(0, dk[lo:lo + step].long(), w[lo:lo + step])
    return out.cpu().numpy()


def dense_full(ctx, n, G, values, nonfinite, seed, label):
    import torch

    need_host_gb(n * 12 / 2**30 * 1.6 + 2)
    dk = torch.empty(n, dtype=torch.int32, device="cuda")
    dv = torch.empty(n, dtype=torch.float64, device="cuda")
    ctx.gen_keys_uniform(dk, G, seed)
    kind, a, b = values
    (ctx.gen_values_uniform if kind == "uniform" else ctx.gen_values_normal)(dv, a, b, seed)
    if nonfinite:
        ctx.gen_inject_nonfinite(dv, nonfinite[0], nonfinite[1], seed)
    got = to_host(ctx.groupby_dense(dk, dv, G))
    absum = dense_absum(dk, dv, G)
    keys, vals = dk.cpu().numpy(), dv.cpu().numpy()
    del dk, dv
    torch.cuda.empty_cache()
    want = oracle.moments_grouped_mt(vals, keys, G, threads=threads())
    check(got, want, absum, label)
    return want


def test_low_cardinality_full_size(ctx):
    want = dense_full(ctx, 1_000_000_000, 256, ("uniform", -1.0, 1.0), None, 0, "1e9 rows x 256 groups")
    assert want["counts"].sum() == 1_000_000_000


def test_numerical_stress_full_size(ctx):
    want = dense_full(ctx, 200_000_000, 10_000, ("normal", 1e9, 1e-3), (0.01, 0.001), 0,
                      "2e8 rows x 10000 groups, NaN / inf")
    assert 0 < want["counts"].sum() < 200_000_000  # NaN rows are not counted


def oracle_i64_buckets(keys_d, v_d, nb):
    """oracle.groupby_i64 over nb key-disjoint buckets in parallel threads: rows permuted on the
    device by a hash of their key (exact sums do not depend on row order).  Returns the
    concatenated (keys, counts, sums, m2s)."""
    import torch

    b = ((keys_d * -7046029254386353131) >> 40) % nb
    order = torch.argsort(b, stable=True)
    counts = torch.bincount(b, minlength=nb).cpu().numpy()
    k = keys_d[order].cpu().numpy()
    v = v_d[order].cpu().numpy()
    del order, b
    cuts = np.concatenate([[0], np.cumsum(counts)])
    res = [None] * nb

    def work(t):
        res[t] = oracle.groupby_i64(k[cuts[t]:cuts[t + 1]], v[cuts[t]:cuts[t + 1]])

    ths = [threading.Thread(target=work, args=(t,)) for t in range(nb)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    return {f: np.concatenate([r[f] for r in res]) for f in ("keys", "counts", "sums", "m2s")}


def compare_i64(gk, got, want, keys_d, v_d, label, with_m2):
    """Same group set; counts bit-exact, sums within 1e-12 * sum|x|, mean = sum / count, m2 within
    1e-9 relative -- compared on the device after sorting both sides by key."""
    import torch

    dev = gk.device
    ok_keys, perm_w = torch.sort(torch.as_tensor(want["keys"]).to(dev))
    my_keys, perm_g = torch.sort(gk)
    assert torch.equal(ok_keys, my_keys), f"{label}: group keys differ ({gk.numel()} vs {ok_keys.numel()})"
    g = ok_keys.numel()

    def mine(f):
        return got[f][perm_g]

    def theirs(f):
        return torch.as_tensor(want[f]).to(dev)[perm_w]

    assert torch.equal(mine("count"), theirs("counts")), f"{label} count"
    absum = torch.zeros(g, dtype=torch.float64, device=dev)
    step = 1 << 27
    zero = torch.zeros((), dtype=torch.float64, device=dev)
    for lo in range(0, keys_d.numel(), step):
        kk, vv = keys_d[lo:lo + step], v_d[lo:lo + step]
        gi = torch.searchsorted(ok_keys, kk)
        absum.index_add_(0, gi, torch.where(torch.isfinite(vv), vv.abs(), zero))
    err = (mine("sum") - theirs("sums")).abs()
    assert bool(torch.all(err <= SUM_TOL * absum)), f"{label} sum: worst {float((err - SUM_TOL * absum).max())}"
    c = mine("count")
    mean_w = torch.where(c > 0, theirs("sums") / torch.where(c > 0, c, torch.ones_like(c)),
                         torch.full_like(c, float("nan")))
    okm = torch.where(c > 0, (mine("mean") - mean_w).abs() <= SUM_TOL * absum / c.clamp(min=1),
                      torch.isnan(mine("mean")))
    assert bool(torch.all(okm)), f"{label} mean"
    if with_m2:
        w = theirs("m2s")
        assert bool(torch.all((mine("m2") - w).abs() <= 1e-9 * w.abs())), f"{label} m2"


def test_fused_pipeline_full_size(ctx):
    import torch

    need_host_gb(6)
    n, ids, seed = 100_000_000, 1_000_000, 0
    dk = torch.empty(n, dtype=torch.int64, device="cuda")
    ctx.gen_keys_cdf(dk, torch.as_tensor(oracle.zipf_cdf(ids, 1.1)).cuda(), SALT, seed)
    cols = []
    for j in (1, 2, 3):
        t = torch.empty(n, dtype=torch.float64, device="cuda")
        ctx.gen_values_normal(t, 0.0, 1.0, seed + j)
        cols.append(t)
    gk, out = ctx.groupby_hash(dk, cols[0], ids, b=cols[1], c=cols[2], expr="a*b+c", pred=">", threshold=0.0,
                               fields=("count", "sum", "mean", "m2", "var_pop", "var_samp"))
    # the oracle's value column and row selection, on the host bytes of the same columns
    a, b, c = (t.cpu().numpy() for t in cols)
    v = oracle.map2("a + b", oracle.map2("a * b", a, b), c)
    m = oracle.filter_mask("gt", 0.0, a)
    live = ((m[np.arange(n) // 64] >> (np.arange(n) % 64).astype(np.uint64)) & np.uint64(1)).astype(bool)
    keys_l = torch.as_tensor(dk.cpu().numpy()[live]).cuda()
    v_l = torch.as_tensor(v[live]).cuda()
    del cols, a, b, c
    want = oracle_i64_buckets(keys_l, v_l, threads())
    compare_i64(gk, out, want, keys_l, v_l, "pipeline 1e8 rows", with_m2=True)


def test_high_cardinality_real_key_space(ctx):
    import torch

    import winrapids_b200 as wb

    need_host_gb(30)
    n, ids, seed = 250_000_000, 1 << 28, 0
    dk = torch.empty(n, dtype=torch.int64, device="cuda")
    dv = torch.empty(n, dtype=torch.float32, device="cuda")
    ctx.gen_keys_ids(dk, ids, SALT, seed)
    ctx.gen_values_lognormal_f32(dv, 0.0, 1.0, seed)
    gk, out = ctx.groupby_hash(dk, dv, ids, fields=wb.SUMCOUNT_FIELDS)
    assert gk.numel() > 150_000_000  # about 2^28 * (1 - exp(-n / 2^28)) distinct keys
    v64 = dv.double()
    del dv
    want = oracle_i64_buckets(dk, v64, threads())
    compare_i64(gk, out, want, dk, v64, "2.5e8 rows over 2^28 ids", with_m2=False)
