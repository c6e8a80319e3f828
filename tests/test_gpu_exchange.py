"""The sharded dense groupby with its exchange over NVLink peer memory (tbgb_groupby_dense_sharded),
on two GPUs, one process each: results against the oracle over several epochs, and the bounded
wait when a rank never pushes (the other rank's merge gives up and reports TBGB_ERR_TIMEOUT; no
rank is left with kernels in flight).  Needs two GPUs: skipped otherwise."""
import os
import socket

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

WORLD = 2


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime

    import torch
    import torch.distributed as dist

    import winrapids_b200 as wb
    from winrapids_b200.sharded import PeerShardedDenseGroupby

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    ctx = wb.Context(rank)
    sh = None
    try:
        n, G = 3_000_017, 256
        lo, hi = n * rank // WORLD, n * (rank + 1) // WORLD
        out = ctx.alloc_moments(G, wb.MOMENT_FIELDS + (("m3", "m4") if mode == "m34" else ()))
        sh = PeerShardedDenseGroupby(ctx, dist, WORLD, rank, G, out, f"cuda:{rank}")
        results = []
        for seed in (1, 2, 3):
            keys = oracle.gen_keys_uniform(n, G, seed)
            vals = oracle.gen_values_normal(n, 0.0, 1.0, seed)
            vals[::97] = 0.0
            vals[::101] = -0.0
            vals[::1009] = np.inf
            vals[::1013] = np.nan
            if mode == "timeout" and rank == 1 and seed == 2:
                break  # rank 1 leaves between steps: rank 0's second merge must give up
            sh.step(torch.from_numpy(keys[lo:hi]).cuda(), torch.from_numpy(vals[lo:hi]).cuda(), lo)
            try:
                ctx.sync()
                results.append({f: t.cpu().numpy().copy() for f, t in out.items()})
            except wb.TambearGbError as e:
                results.append(e.kind)
                break
        q.put((rank, results))
        dist.barrier()
        sh.finish()  # unmap, wait until no rank maps this rank's buffer, free it
        sh = None
    finally:
        if sh is not None:
            sh.close()
        ctx.close()
        dist.destroy_process_group()


def _spawn(mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return sorted(res, key=lambda x: x[0])


def _need_two_gpus():
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")


@pytest.mark.parametrize("mode", ["ok", "m34"])
def test_peer_exchange_matches_oracle(mode):
    """Without m3 / m4 among the outputs the shards' states skip them; with them they travel too."""
    _need_two_gpus()
    from parity import abs_sums, check
    from test_gpu_higher_moments import check_m34

    res = _spawn(mode)
    n, G = 3_000_017, 256
    for i, seed in enumerate((1, 2, 3)):
        keys = oracle.gen_keys_uniform(n, G, seed)
        vals = oracle.gen_values_normal(n, 0.0, 1.0, seed)
        vals[::97] = 0.0
        vals[::101] = -0.0
        vals[::1009] = np.inf
        vals[::1013] = np.nan
        want = oracle.moments_grouped_mt(vals, keys, G, threads=8, m34=mode == "m34")
        for rank, results in res:  # every rank holds the merged result of every epoch
            check(results[i], want, abs_sums(keys, vals, G), f"rank {rank} epoch {i + 1}")
            if mode == "m34":
                check_m34(results[i], want, keys, vals, G, f"rank {rank} epoch {i + 1}")


@pytest.mark.parametrize("m34", [False, True])
def test_sharded_entry_one_rank(ctx, m34):
    """tbgb_groupby_dense_sharded with one rank (no peers): the shard's state table goes through
    the exchange buffer and the merge, over several epochs, with and without m3 / m4."""
    import torch

    import winrapids_b200 as wb
    from parity import abs_sums, check
    from test_gpu_higher_moments import check_m34

    n, G = 1_000_003, 300
    own = ctx.exchange_alloc(1, G)
    try:
        for epoch, seed in enumerate((4, 5, 6), start=1):
            keys = oracle.gen_keys_uniform(n, G, seed)
            vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 3.0, 2.0, seed), 0.01, 0.002, seed)
            out = ctx.alloc_moments(G, wb.MOMENT_FIELDS + (("m3", "m4") if m34 else ()))
            ctx.groupby_dense_sharded(torch.from_numpy(keys).cuda(), torch.from_numpy(vals).cuda(), G, 0, 0, [own],
                                      epoch, out)
            ctx.sync()
            got = {f: t.cpu().numpy() for f, t in out.items()}
            want = oracle.moments_grouped_mt(vals, keys, G, threads=8, m34=m34)
            check(got, want, abs_sums(keys, vals, G), f"epoch {epoch}")
            if m34:
                check_m34(got, want, keys, vals, G, f"epoch {epoch}")
    finally:
        ctx.exchange_free(own)


def test_peer_exchange_wait_is_bounded():
    _need_two_gpus()
    res = _spawn("timeout")
    r0, r1 = res[0][1], res[1][1]
    assert isinstance(r0[0], dict) and isinstance(r1[0], dict)   # epoch 1 completes on both
    assert r0[1] == "Timeout" and len(r1) == 1                   # rank 0 gives up on epoch 2
