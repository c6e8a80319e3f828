"""GPU tests of the owner routing (tbgb_hash_partition) and of the sharded int64-key path
emulated on one GPU (shards partitioned, parts concatenated per owner in shard order,
each owner grouped), against the oracle."""
import numpy as np
import pytest

import oracle
from parity import to_host
from test_gpu_table import dev, dev_mask, hash_check, host_mask, host_value, rows_of

pytestmark = pytest.mark.gpu

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def fmix64_np(k):
    k = np.asarray(k).view(np.uint64).copy()
    with np.errstate(over="ignore"):
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xFF51AFD7ED558CCD)
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xC4CEB9FE1A85EC53)
        k ^= k >> np.uint64(33)
    return k


def owner_np(keys, P):
    return ((fmix64_np(keys) >> np.uint64(32)) % np.uint64(P)).astype(np.int64)


def run_partition(ctx, keys, a, P, b=None, c=None, expr="a", pred=None, thr=0.0, mask=None):
    import torch

    n = keys.size
    pk = torch.empty(max(n, 1), dtype=torch.int64, device="cuda")
    pv = torch.empty(max(n, 1), dtype=torch.float64, device="cuda")
    pc = torch.zeros(P, dtype=torch.int64, device="cuda")
    ctx.hash_partition(dev(keys), dev(a), P, pk, pv, pc, b=None if b is None else dev(b),
                       c=None if c is None else dev(c), expr=expr, pred=pred, threshold=thr, mask=dev_mask(mask))
    ctx.sync()
    return pk.cpu().numpy(), pv.cpu().numpy(), pc.cpu().numpy()


@pytest.mark.parametrize("P", [1, 2, 3, 8, 32])
@pytest.mark.parametrize("f32", [False, True])
def test_partition_is_stable_and_complete(ctx, P, f32):
    rng = np.random.default_rng(P)
    n = 300_007
    keys = rng.integers(-2**63, 2**63 - 1, n, dtype=np.int64)
    keys[::101] = np.iinfo(np.int64).min
    a = rng.normal(size=n)
    b = rng.normal(size=n)
    c = rng.normal(size=n)
    a[::97] = np.nan
    if f32:
        a, b, c = a.astype(np.float32), b.astype(np.float32), c.astype(np.float32)
    user = host_mask(n)
    user[::4] = np.uint64(0x00FF00FF00FF00FF)
    pk, pv, pc = run_partition(ctx, keys, a, P, b, c, expr="a*b+c", pred="<=", thr=0.3, mask=user)
    m = host_mask(n, np.asarray(a, np.float64), "<=", 0.3, user)
    live = rows_of(m, n)
    v = host_value(a, b, c, "a*b+c")
    own = owner_np(keys, P)
    start = 0
    for p in range(P):
        sel = live & (own == p)
        cnt = int(sel.sum())
        assert pc[p] == cnt, (p, pc[p], cnt)
        assert np.array_equal(pk[start:start + cnt], keys[sel]), f"part {p} keys"
        assert np.array_equal(pv[start:start + cnt].view(np.uint64), v[sel].view(np.uint64)), f"part {p} values"
        start += cnt
    assert start == int(live.sum())


def test_partition_empty(ctx):
    pk, pv, pc = run_partition(ctx, np.zeros(0, np.int64), np.zeros(0), 4)
    assert np.all(pc == 0)


@pytest.mark.parametrize("R", [2, 4])
def test_sharded_hash_groupby_emulated(ctx, R):
    """R shards routed to R owners; every owner groups the rows it receives (senders in shard
    order); the union of the owners' groups equals the unsharded oracle groupby, extrema
    (with +-0 ties in global row order) bit-exact."""
    import torch

    n, ids, seed = 1_200_000, 300_000, 8
    keys = oracle.gen_keys_ids(n, ids, 0x1234, seed)
    rng = np.random.default_rng(seed)
    a = rng.normal(size=n)
    a[rng.random(n) < 0.02] = 0.0
    a[rng.random(n) < 0.02] = -0.0
    a[rng.random(n) < 0.01] = np.nan
    a[rng.random(n) < 0.005] = np.inf
    bounds = np.linspace(0, n, R + 1).astype(np.int64)
    parts = []
    for r in range(R):
        lo, hi = bounds[r], bounds[r + 1]
        pk, pv, pc = run_partition(ctx, keys[lo:hi], a[lo:hi], R)
        offs = np.concatenate([[0], np.cumsum(pc)])
        parts.append([(pk[offs[p]:offs[p + 1]], pv[offs[p]:offs[p + 1]]) for p in range(R)])
    all_keys, all_out = [], []
    for owner in range(R):
        rk = np.concatenate([parts[r][owner][0] for r in range(R)])
        rv = np.concatenate([parts[r][owner][1] for r in range(R)])
        gk, out = ctx.groupby_hash(dev(rk), dev(rv), ids)
        all_keys.append(gk.cpu().numpy())
        all_out.append(to_host(out))
    gk = np.concatenate(all_keys)
    got = {f: np.concatenate([o[f] for o in all_out]) for f in all_out[0]}
    assert np.unique(gk).size == gk.size, "a key owned by two ranks"
    want = oracle.groupby_i64(keys, a)
    hash_check(gk, got, want, a, keys, None, f"sharded R={R}")
