"""The parity check bench.py runs after its timed region (the `check` field of the JSON line),
on CPU tensors: it passes on results the oracle produced for the same rows, fails on a planted
mistake, and gives the same answer when the rows are split over two gloo ranks."""
import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
import oracle


def _dense_case(n=200_000, G=37, seed=3):
    keys = oracle.gen_keys_uniform(n, G, seed)
    vals = oracle.inject_nonfinite(oracle.gen_values_normal(n, 1e9, 1e-3, seed), 0.01, 0.002, seed)
    vals[5::9001] = 0.0
    want = oracle.moments_grouped_mt(vals, keys, G, threads=4)
    d = oracle.derived(want)
    out = {"count": want["counts"], "sum": want["sums"], "min": want["mins"], "max": want["maxs"],
           "mean": d["mean"], "m2": want["m2s"], "var_pop": d["var_pop"], "var_samp": d["var_samp"]}
    return keys, vals, {f: torch.from_numpy(np.ascontiguousarray(v)) for f, v in out.items()}, G


def test_dense_check_accepts_the_oracle_and_rejects_planted_mistakes():
    keys, vals, out, G = _dense_case()
    k, v = torch.from_numpy(keys), torch.from_numpy(vals)
    r = bench.dense_check(k, v, out, G, None)
    assert r["ok"], r
    for f, bad in (("count", lambda t: t.__setitem__(3, t[3] + 1)),
                   ("min", lambda t: t.__setitem__(4, np.nextafter(t[4].item(), 0.0))),
                   ("sum", lambda t: t.__setitem__(5, t[5] * (1 + 1e-9))),
                   ("m2", lambda t: t.__setitem__(6, t[6] * (1 + 1e-7)))):
        o = {x: y.clone() for x, y in out.items()}
        bad(o[f])
        r = bench.dense_check(k, v, o, G, None)
        assert not r["ok"] and not r["fields"][f], (f, r)


def _hash_case(n=300_000, ids=50_000, seed=4):
    keys = oracle.gen_keys_ids(n, ids, 0x5EED5EED12345678, seed)
    vals = oracle.gen_values_lognormal_f32(n, 0.0, 1.0, seed)
    want = oracle.groupby_i64(keys, vals.astype(np.float64))
    g = want["keys"].size
    out = {"count": torch.from_numpy(want["counts"]), "sum": torch.from_numpy(want["sums"]),
           "mean": torch.from_numpy(want["sums"] / want["counts"])}
    job = SimpleNamespace(ng=torch.tensor([g]), out_keys=torch.from_numpy(want["keys"]), out=out, op={})
    return keys, vals, job


def test_hash_check_accepts_the_oracle_and_rejects_planted_mistakes():
    keys, vals, job = _hash_case()
    dev_in = [torch.from_numpy(keys), torch.from_numpy(vals)]
    r = bench.hash_check(job, dev_in, None, 1)
    assert r["ok"], r
    job.out["count"][7] += 1  # a row counted in the wrong group
    job.out["count"][8] -= 1
    r = bench.hash_check(job, dev_in, None, 1)
    assert not r["ok"] and not r["fields"]["count"], r
    job.out["count"][7] -= 1
    job.out["count"][8] += 1
    job.out_keys[9] = job.out_keys[10]  # a key reported twice
    r = bench.hash_check(job, dev_in, None, 1)
    assert not r["ok"] and not r["fields"]["unique"], r


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        keys, vals, out, G = _dense_case()
        n = keys.size
        lo, hi = n * rank // world, n * (rank + 1) // world
        r = bench.dense_check(torch.from_numpy(keys[lo:hi]), torch.from_numpy(vals[lo:hi]), out, G, dist)
        # int64 keys: each rank holds the groups of the keys it owns (by a split of its own here)
        hk, hv, job = _hash_case()
        own = (np.asarray(job.out_keys) % world) == rank
        job.out_keys = job.out_keys[own].clone()
        job.out = {f: t[own].clone() for f, t in job.out.items()}
        job.ng = torch.tensor([int(own.sum())])
        hlo, hhi = hk.size * rank // world, hk.size * (rank + 1) // world
        h = bench.hash_check(job, [torch.from_numpy(hk[hlo:hhi]), torch.from_numpy(hv[hlo:hhi])], dist, world)
        # the same key owned by both ranks is caught
        job.out_keys[0] = 12345
        h2 = bench.hash_check(job, [torch.from_numpy(hk[hlo:hhi]), torch.from_numpy(hv[hlo:hhi])], dist, world)
        q.put((rank, r["ok"], h["ok"], h2["ok"]))
    finally:
        dist.destroy_process_group()


def test_checks_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=5) for _ in range(2))
    assert [g[1:] for g in got] == [(True, True, False), (True, True, False)], got
