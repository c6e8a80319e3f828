"""The owner-sharded int64-key groupby (winrapids_b200.sharded.ShardedHashGroupby) on two GPUs,
one process each over NCCL: every rank routes its rows to the owner of their key, the parts cross
NVLink (one NCCL all-to-all, or the owner's second radix pass reading the senders' buffers in
place through peer memory), and each owner groups its keys.  The union of the ranks' groups
must equal the oracle's groupby of all rows (each key on exactly one rank; counts bit-exact, sums
within 1e-12 * sum|x|), for the high-cardinality shape (f32 values) and the fused pipeline shape
(filter a > 0, v = a*b + c).  Needs two GPUs: skipped otherwise."""
import os
import socket

import numpy as np
import pytest

import oracle
from parity import SUM_TOL

pytestmark = pytest.mark.gpu

WORLD = 2
SALT = 0x5EED5EED12345678


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(shape, n):
    if shape == "highcard":
        keys = oracle.gen_keys_ids(n, 1 << 20, SALT, 7)
        return keys, [oracle.gen_values_lognormal_f32(n, 0.0, 1.0, 7)]
    keys = oracle.gen_keys_cdf(n, oracle.zipf_cdf(100_000, 1.1), SALT, 8)
    return keys, [oracle.gen_values_normal(n, 0.0, 1.0, 8 + j) for j in (1, 2, 3)]


def _worker(rank, port, shape, exchange, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime

    import torch
    import torch.distributed as dist

    import winrapids_b200 as wb
    from winrapids_b200.sharded import ShardedHashGroupby

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    ctx = wb.Context(rank)
    try:
        n = 4_000_037
        lo, hi = n * rank // WORLD, n * (rank + 1) // WORLD
        keys, cols = _inputs(shape, n)
        dcols = [torch.from_numpy(c[lo:hi]).cuda() for c in cols]
        sh = ShardedHashGroupby(ctx, dist, WORLD, hi - lo, 1 << 20, wb.SUMCOUNT_FIELDS, f"cuda:{rank}",
                                exchange=exchange)
        kw = {} if shape == "highcard" else dict(b=dcols[1], c=dcols[2], expr="a*b+c", pred=">", threshold=0.0)
        for _ in range(2):  # the second step reuses every buffer
            sh.step(torch.from_numpy(keys[lo:hi]).cuda(), dcols[0], **kw)
        gk, out = sh.result()
        q.put((rank, gk.cpu().numpy(), {f: t.cpu().numpy() for f, t in out.items()}))
        sh.finish()
        dist.barrier()
    finally:
        ctx.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "pull"])
@pytest.mark.parametrize("shape", ["highcard", "pipeline"])
def test_sharded_hash_groupby_matches_oracle(shape, exchange):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    spawn = mp.get_context("spawn")
    q = spawn.Queue()
    port = free_port()
    procs = [spawn.Process(target=_worker, args=(r, port, shape, exchange, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(WORLD)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    n = 4_000_037
    keys, cols = _inputs(shape, n)
    if shape == "highcard":
        v = cols[0].astype(np.float64)
        mask = None
    else:
        v = oracle.map2("a + b", oracle.map2("a * b", cols[0], cols[1]), cols[2])
        mask = oracle.filter_mask("gt", 0.0, cols[0])
    want = oracle.groupby_i64(keys, v, mask=mask)
    gk = np.concatenate([r[1] for r in res])
    assert np.unique(gk).size == gk.size, "a key is held by both ranks"
    order = np.argsort(gk)
    wo = np.argsort(want["keys"])
    assert np.array_equal(gk[order], want["keys"][wo])
    cnt = np.concatenate([r[2]["count"] for r in res])[order]
    s = np.concatenate([r[2]["sum"] for r in res])[order]
    assert np.array_equal(cnt, want["counts"][wo])
    live = np.ones(n, bool) if mask is None else \
        ((mask[np.arange(n) // 64] >> (np.arange(n) % 64).astype(np.uint64)) & np.uint64(1)).astype(bool)
    sk = want["keys"][wo]
    gi = np.searchsorted(sk, keys[live])
    absum = np.bincount(gi, weights=np.abs(v[live]), minlength=sk.size)
    assert np.all(np.abs(s - want["sums"][wo]) <= SUM_TOL * absum)
