"""The owner-sharded radix groupby's two halves on one GPU, the ranks emulated: W shards are each
routed (tbgb_radix_route), and every owner groups its digits reading the shards' routed rows in
place -- one start address per sender, as the peer-memory exchange passes them -- through
tbgb_radix_groupby_routed.  The union of the owners' groups must equal the oracle's groupby of all
rows (each key on exactly one owner); also with mask + predicate + expression, with empty senders,
and with a heavy key whose bucket overflows (the gated global-table fallback then reads every
sender's block)."""
import numpy as np
import pytest

import oracle
from parity import SUM_TOL, abs_sums

pytestmark = pytest.mark.gpu
SALT = 0x5EED5EED12345678


def fmix64(k):
    m = (1 << 64) - 1
    x = k & m
    x ^= x >> 33
    x = (x * 0xFF51AFD7ED558CCD) & m
    x ^= x >> 33
    x = (x * 0xC4CEB9FE1A85EC53) & m
    return x ^ (x >> 33)


def owned_digits(world):
    return [(512 * r + world - 1) // world for r in range(world + 1)]


def run_emulated(ctx, keys, cols, world, op=None, fallback=None, empty_sender=None):
    """fallback: the fallback bits each owner must report (default: none falls back)."""
    import torch

    import winrapids_b200 as wb

    n = keys.size
    op = op or {}
    fallback = fallback or [0] * world
    lo = owned_digits(world)
    bounds = [n * r // world for r in range(world + 1)]
    if empty_sender is not None:  # one shard without rows
        bounds[empty_sender + 1] = bounds[empty_sender]
    routed, counts = [], []
    vb = None
    for s in range(world):
        a, b = bounds[s], bounds[s + 1]
        dk = torch.from_numpy(np.ascontiguousarray(keys[a:b])).cuda()
        dc = [torch.from_numpy(np.ascontiguousarray(c[a:b])).cuda() for c in cols]
        kw = dict(op)
        if "mask" in kw:  # the shard's own mask words (shards start on 64-row boundaries here)
            assert a % 64 == 0
            kw["mask"] = kw["mask"][a // 64:(b + 63) // 64]
        bcol = dc[1] if len(dc) > 1 else None
        ccol = dc[2] if len(dc) > 2 else None
        vb = ctx.radix_value_bytes(dc[0], bcol, ccol, kw.get("expr", "a"), kw.get("pred"), kw.get("threshold", 0.0))
        h = torch.empty(max(b - a, 1), dtype=torch.int64, device="cuda")
        v = torch.empty(max(b - a, 1), dtype=torch.float32 if vb == 4 else torch.float64, device="cuda")
        d = torch.zeros(512, dtype=torch.int64, device="cuda")
        ctx.radix_route(dk, dc[0], h, v, d, b=bcol, c=ccol, **kw)
        routed.append((h, v))
        counts.append(d)
    ctx.sync()
    table = torch.stack(counts).cpu().numpy()
    got_keys, got = [], {"count": [], "sum": []}
    for q in range(world):
        nd = lo[q + 1] - lo[q]
        seg = torch.from_numpy(np.ascontiguousarray(table[:, lo[q]:lo[q + 1]]).reshape(-1)).cuda()
        before = table[:, :lo[q]].sum(1)
        rows = [int(x) for x in table[:, lo[q]:lo[q + 1]].sum(1)]
        hashes = [int(routed[s][0].data_ptr()) + 8 * int(before[s]) for s in range(world)]
        vals = [int(routed[s][1].data_ptr()) + vb * int(before[s]) for s in range(world)]
        mg = 1 << 20
        ok = torch.empty(mg, dtype=torch.int64, device="cuda")
        out = {f: torch.empty(mg, dtype=torch.float64, device="cuda") for f in wb.SUMCOUNT_FIELDS}
        ng = torch.zeros(1, dtype=torch.int64, device="cuda")
        ctx.radix_groupby_routed(hashes, vals, rows, seg, lo[q], nd, mg, ok, out, ng, value_bytes=vb)
        bits = ctx.radix_fallback()
        assert bits == fallback[q], f"owner {q}: fallback bits {bits}, expected {fallback[q]}"
        g = int(ng.item())
        got_keys.append(ok[:g].cpu().numpy())
        for f in got:
            got[f].append(out[f][:g].cpu().numpy())
    return np.concatenate(got_keys), {f: np.concatenate(x) for f, x in got.items()}


def check(gk, got, keys, v, live):
    assert np.unique(gk).size == gk.size, "a key is held by two owners"
    want = oracle.groupby_i64(keys[live], v[live])
    order = np.argsort(gk, kind="stable")
    assert np.array_equal(gk[order], want["keys"])
    assert np.array_equal(got["count"][order], want["counts"])
    codes = np.searchsorted(want["keys"], keys[live])
    absum = abs_sums(codes, v[live], want["keys"].size)
    assert np.all(np.abs(got["sum"][order] - want["sums"]) <= SUM_TOL * absum)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_routed_f32_in_place(ctx, world):
    n = 3_000_064
    keys = oracle.gen_keys_ids(n, 1 << 19, SALT, 21)
    vals = oracle.gen_values_lognormal_f32(n, 0.0, 1.0, 21)
    gk, got = run_emulated(ctx, keys, [vals], world)
    check(gk, got, keys, vals.astype(np.float64), np.ones(n, bool))


def test_routed_masked_expression_and_an_empty_sender(ctx):
    import torch

    n = 2_000_128  # shards of 500,032 rows: each starts on a 64-row mask word
    keys = oracle.gen_keys_ids(n, 1 << 18, SALT, 22)
    a = oracle.gen_values_normal(n, 0.0, 1.0, 22)
    b = oracle.gen_values_normal(n, 1.0, 1.0, 23)
    c = oracle.gen_values_normal(n, 0.0, 2.0, 24)
    rng = np.random.default_rng(25)
    live_mask = rng.random(n) < 0.6
    words = np.zeros((n + 63) // 64, dtype=np.uint64)
    idx = np.nonzero(live_mask)[0]
    np.bitwise_or.at(words, idx // 64, np.left_shift(np.uint64(1), (idx % 64).astype(np.uint64)))
    op = dict(expr="a*b+c", pred=">", threshold=-0.25, mask=torch.from_numpy(words.view(np.int64)).cuda())
    gk, got = run_emulated(ctx, keys, [a, b, c], 4, op=op, empty_sender=2)
    v = oracle.map2("a + b", oracle.map2("a * b", a, b), c)
    check(gk, got, keys, v, live_mask & (a > -0.25))


def test_routed_heavy_key_falls_back_over_every_sender(ctx):
    n = 2_000_000
    keys = oracle.gen_keys_ids(n, 1 << 18, SALT, 26)
    keys[np.random.default_rng(26).random(n) < 0.5] = 77  # one key on half the rows
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 26)
    digit = int(fmix64(77) >> 55)
    owner = 0 if digit < owned_digits(2)[1] else 1
    gk, got = run_emulated(ctx, keys, [vals], 2, fallback=[1 if q == owner else 0 for q in range(2)])
    check(gk, got, keys, vals, np.ones(n, bool))
