"""Host logic of the row-sharded paths (winrapids_b200.sharded) on world_size-2 gloo
process groups, CPU only.  The GPU kernels are stood in for by oracle-based fakes with
the same methods as winrapids_b200.Context, so what is tested is the collective
choreography: split sizes, rank order of the exchanged parts, state gathering and
folding order, and that a rank whose receive buffer is too small fails on every rank
instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle

WORLD = 2


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def fmix64_np(keys):
    k = np.asarray(keys).view(np.uint64).copy()
    with np.errstate(over="ignore"):
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xFF51AFD7ED558CCD)
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xC4CEB9FE1A85EC53)
        k ^= k >> np.uint64(33)
    return k


def unfmix64_np(h):
    inv = lambda c: pow(c, -1, 1 << 64)  # noqa: E731
    x = np.asarray(h, dtype=np.uint64).copy()
    with np.errstate(over="ignore"):
        x ^= x >> np.uint64(33)
        x *= np.uint64(inv(0xC4CEB9FE1A85EC53))
        x ^= x >> np.uint64(33)
        x *= np.uint64(inv(0xFF51AFD7ED558CCD))
        x ^= x >> np.uint64(33)
    return x.view(np.int64)


def radix_owner_np(keys, P):
    d = (fmix64_np(keys) >> np.uint64(55)).astype(np.int64)
    return d * P // 512


def owner_np(keys, P):
    k = np.asarray(keys).view(np.uint64).copy()
    with np.errstate(over="ignore"):
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xFF51AFD7ED558CCD)
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xC4CEB9FE1A85EC53)
        k ^= k >> np.uint64(33)
    return ((k >> np.uint64(32)) % np.uint64(P)).astype(np.int64)


class FakeCtx:
    """CPU stand-in for winrapids_b200.Context: same method names and buffer contracts."""

    # hash path ------------------------------------------------------------------------
    def hash_partition(self, keys, a, n_parts, out_keys, out_vals, part_counts, b=None, c=None, expr="a",
                       pred=None, threshold=0.0, mask=None):
        k = keys.numpy()
        v = a.numpy().astype(np.float64)
        own = owner_np(k, n_parts)
        order = np.argsort(own, kind="stable")
        out_keys[:k.size] = torch.from_numpy(k[order])
        out_vals[:k.size] = torch.from_numpy(v[order])
        part_counts[:] = torch.from_numpy(np.bincount(own, minlength=n_parts).astype(np.int64))

    def groupby_hash_into(self, keys, a, max_groups, out_keys, out, n_groups, **kw):
        res = oracle.groupby_i64(keys.numpy(), a.numpy().astype(np.float64))
        g = res["keys"].size
        out_keys[:g] = torch.from_numpy(res["keys"])
        out["count"][:g] = torch.from_numpy(res["counts"])
        out["sum"][:g] = torch.from_numpy(res["sums"])
        n_groups[0] = g

    # radix routing -----------------------------------------------------------------------
    def radix_value_bytes(self, a, b=None, c=None, expr="a", pred=None, threshold=0.0):
        return 4 if a.dtype == torch.float32 and expr == "a" else 8

    def radix_route(self, keys, a, out_hashes, out_vals, digit_counts, b=None, c=None, expr="a", pred=None,
                    threshold=0.0, mask=None):
        h = fmix64_np(keys.numpy())
        d = (h >> np.uint64(55)).astype(np.int64)
        order = np.argsort(d, kind="stable")
        m = h.size
        out_hashes[:m] = torch.from_numpy(h[order].view(np.int64))
        out_vals[:m] = a[torch.from_numpy(order)]
        digit_counts[:] = torch.from_numpy(np.bincount(d, minlength=512).astype(np.int64))

    def radix_groupby_routed(self, hashes, vals, sender_rows, seg_counts, digit_lo, n_digits, max_groups,
                             out_keys, out, n_groups, value_bytes=None):
        assert value_bytes in (None, vals.element_size())
        n_senders, n_rows = len(sender_rows), sum(sender_rows)
        h = hashes[:n_rows].numpy().view(np.uint64)
        d = (h >> np.uint64(55)).astype(np.int64)
        assert np.all((d >= digit_lo) & (d < digit_lo + n_digits)), "a row routed to a rank that does not own it"
        # the blocks are in sender order, each in digit order, with the announced sizes
        sizes = seg_counts.numpy().reshape(n_senders, n_digits)
        assert sizes.sum() == n_rows and list(sizes.sum(1)) == list(sender_rows)
        exp = np.concatenate([np.repeat(np.arange(digit_lo, digit_lo + n_digits), sizes[s]) for s in range(n_senders)])
        assert np.array_equal(d, exp)
        res = oracle.groupby_i64(unfmix64_np(h), vals[:n_rows].numpy().astype(np.float64))
        g = res["keys"].size
        out_keys[:g] = torch.from_numpy(res["keys"])
        out["count"][:g] = torch.from_numpy(res["counts"])
        out["sum"][:g] = torch.from_numpy(res["sums"])
        n_groups[0] = g

    def sync(self):
        pass

    # dense path: state = (count, exact sum, min, max) per group, folded in rank order --
    def state_bytes(self, G):
        return 4 * G * 8

    def groupby_dense_state(self, keys, vals, G, row_offset=0, mask=None, state=None):
        st = oracle.moments_grouped_mt(vals.numpy(), keys.numpy(), G, threads=1)
        s = state.view(4, G)
        for i, f in enumerate(("counts", "sums", "mins", "maxs")):
            s[i] = torch.from_numpy(st[f])

    def merge_states(self, states, n_states, G, out=None):
        s = states.view(n_states, 4, G).numpy()
        out["count"][:] = torch.from_numpy(s[:, 0].sum(axis=0))
        tot = np.zeros(G)
        for r in range(n_states):  # rank order
            tot = tot + s[r, 1]
        out["sum"][:] = torch.from_numpy(tot)
        out["min"][:] = torch.from_numpy(s[:, 2].min(axis=0))
        out["max"][:] = torch.from_numpy(s[:, 3].max(axis=0))


def _init(rank, port, world=WORLD):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _hash_worker(rank, port, n, ids, fields, q):
    from winrapids_b200.sharded import ShardedHashGroupby

    _init(rank, port)
    try:
        keys = oracle.gen_keys_ids(n, ids, 77, 3)
        vals = oracle.gen_values_normal(n, 0.0, 1.0, 3)
        lo, hi = n * rank // WORLD, n * (rank + 1) // WORLD
        sh = ShardedHashGroupby(FakeCtx(), dist, WORLD, hi - lo, ids, fields, "cpu")
        sh.step(torch.from_numpy(keys[lo:hi]), torch.from_numpy(vals[lo:hi]))
        gk, out = sh.result()
        q.put((rank, gk.numpy().copy(), out["count"].numpy().copy(), out["sum"].numpy().copy(), sh.n_recv))
    finally:
        dist.destroy_process_group()


def _small_buffer_worker(rank, port, q):
    from winrapids_b200.sharded import exchange_parts

    _init(rank, port)
    try:
        n = 1000
        pk = torch.arange(n, dtype=torch.int64)
        pv = torch.zeros(n, dtype=torch.float64)
        # rank 0 sends everything to rank 1, whose receive buffer holds 10 rows
        pc = torch.tensor([0, n] if rank == 0 else [0, 0], dtype=torch.int64)
        cap = 10 if rank == 1 else n
        try:
            exchange_parts(dist, pk, pv, pc, torch.empty(cap, dtype=torch.int64), torch.empty(cap), )
            q.put((rank, "no error"))
        except RuntimeError as e:
            q.put((rank, "raised" if "too small" in str(e) else str(e)))
    finally:
        dist.destroy_process_group()


def _dense_worker(rank, port, n, G, q):
    from winrapids_b200.sharded import ShardedDenseGroupby

    _init(rank, port)
    try:
        keys = oracle.gen_keys_uniform(n, G, 5)
        vals = oracle.gen_values_uniform(n, -1.0, 1.0, 5)
        lo, hi = n * rank // WORLD, n * (rank + 1) // WORLD
        out = {f: torch.empty(G, dtype=torch.float64) for f in ("count", "sum", "min", "max")}
        sh = ShardedDenseGroupby(FakeCtx(), dist, WORLD, G, out, "cpu")
        sh.step(torch.from_numpy(keys[lo:hi]), torch.from_numpy(vals[lo:hi]), lo)
        q.put((rank, {f: t.numpy().copy() for f, t in out.items()}))
    finally:
        dist.destroy_process_group()


def _spawn(fn, *args, world=WORLD):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res, key=lambda x: x[0])


@pytest.mark.parametrize("route", ["radix", "stable"])
def test_sharded_hash_groupby_gloo(route):
    """count / sum take the radix routing (digit owners); with min among the outputs the stable
    owner partition runs instead."""
    n, ids = 60_000, 5_000
    fields = ("count", "sum") if route == "radix" else ("count", "sum", "min")
    res = _spawn(_hash_worker, free_port(), n, ids, fields)
    keys = oracle.gen_keys_ids(n, ids, 77, 3)
    vals = oracle.gen_values_normal(n, 0.0, 1.0, 3)
    want = oracle.groupby_i64(keys, vals)
    gk = np.concatenate([r[1] for r in res])
    cnt = np.concatenate([r[2] for r in res])
    sm = np.concatenate([r[3] for r in res])
    assert sum(r[4] for r in res) == n
    own = radix_owner_np if route == "radix" else owner_np
    for rank, k, *_ in res:
        assert np.all(own(k, WORLD) == rank), "a group on a rank that does not own it"
    order = np.argsort(gk)
    assert np.array_equal(gk[order], want["keys"])
    assert np.array_equal(cnt[order], want["counts"])
    # the owner sees each key's rows in global row order, so its exact sums are the oracle's
    assert np.array_equal(sm[order], want["sums"])


def test_exchange_rejects_small_receive_buffer_on_all_ranks():
    res = _spawn(_small_buffer_worker, free_port())
    assert [r[1] for r in res] == ["raised", "raised"]


def test_sharded_dense_gloo():
    n, G = 50_000, 300
    res = _spawn(_dense_worker, free_port(), n, G)
    keys = oracle.gen_keys_uniform(n, G, 5)
    vals = oracle.gen_values_uniform(n, -1.0, 1.0, 5)
    want = oracle.moments_grouped_mt(vals, keys, G, threads=1)
    for _, out in res:  # every rank holds the merged result
        assert np.array_equal(out["count"], want["counts"])
        assert np.array_equal(out["min"], want["mins"]) and np.array_equal(out["max"], want["maxs"])
        absum = np.bincount(keys, weights=np.abs(vals), minlength=G)
        assert np.all(np.abs(out["sum"] - want["sums"]) <= 1e-12 * absum)


# ---- the exchange over peer memory: setup choreography (the kernels need GPUs) ----------

class FakePeerCtx:
    """Stand-in for the exchange-buffer and IPC methods of winrapids_b200.Context: buffers are
    numbers, handles carry the owner's rank; rank `fail_on` cannot map one peer."""

    def __init__(self, rank, fail_on=None):
        self.rank, self.fail_on = rank, fail_on
        self.log = []

    def exchange_alloc(self, world, G):
        self.log.append(("alloc", world, G))
        return 1000 + self.rank

    def exchange_free(self, p):
        self.log.append(("free", p))

    def peer_export(self, p):
        return bytes([self.rank]) * 64

    def peer_import(self, handle):
        if self.rank == self.fail_on:
            raise RuntimeError("cudaIpcOpenMemHandle: mapping refused")
        return 2000 + handle[0]

    def peer_close(self, p):
        self.log.append(("close", p))

    def groupby_dense_sharded(self, keys, vals, G, row_offset, rank, buffers, epoch, out, mask=None):
        self.log.append(("step", tuple(buffers), epoch, row_offset))


def _peer_worker(rank, port, fail_on, world, q):
    from winrapids_b200.sharded import PeerMappingError, PeerShardedDenseGroupby

    _init(rank, port, world)
    try:
        ctx = FakePeerCtx(rank, fail_on)
        try:
            sh = PeerShardedDenseGroupby(ctx, dist, world, rank, 256, {}, "cpu")
        except PeerMappingError as e:
            q.put((rank, "raised", ctx.log, str(e)))
            return
        sh.step(torch.zeros(4, dtype=torch.int32), torch.zeros(4), 10 * rank)
        sh.step(torch.zeros(4, dtype=torch.int32), torch.zeros(4), 10 * rank)
        sh.finish()
        q.put((rank, "ok", ctx.log, ""))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_setup_gloo(world):
    res = _spawn(_peer_worker, free_port(), None, world, world=world)
    for rank, status, log, _ in res:
        assert status == "ok"
        steps = [e for e in log if e[0] == "step"]
        # buffers in rank order: the own buffer at its rank, the peers' mapped ones elsewhere
        want = tuple(1000 + rank if q == rank else 2000 + q for q in range(world))
        assert [s[1] for s in steps] == [want, want]
        assert [s[2] for s in steps] == [1, 2]          # epochs start at 1 and step by one
        closes = [e for e in log if e[0] == "close"]
        assert sorted(closes) == [("close", 2000 + q) for q in range(world) if q != rank]  # every peer unmapped
        assert log[-1] == ("free", 1000 + rank)         # the own buffer freed last


@pytest.mark.parametrize("world,fail_on", [(2, 1), (4, 2)])
def test_peer_exchange_mapping_failure_raises_on_every_rank(world, fail_on):
    res = _spawn(_peer_worker, free_port(), fail_on, world, world=world)
    assert [r[1] for r in res] == ["raised"] * world
    for rank, _, log, msg in res:
        assert ("free", 1000 + rank) in log            # the own buffer released
        assert ("another rank" in msg) == (rank != fail_on)
