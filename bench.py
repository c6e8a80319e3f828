#!/usr/bin/env python
"""Groupby-aggregate throughput on B200: rows/s and HBM GB/s vs the measured peak.

Default workload (the low-cardinality sharded configuration): 1,000,000,000 rows,
int32 keys uniform in [0,256), f64 values ~U(-1,1); count/sum/min/max/mean/var per
key.  Rows are split evenly over N GPUs (one process per GPU, launched by
torch.distributed.run); each GPU reduces its shard to a mergeable per-group state
table and stores it into every other GPU's exchange buffer over NVLink peer memory,
and every GPU folds the tables in rank order (an NCCL all-gather when the peer
mappings cannot be made).

Other workloads (--workload): `pipeline` (100,000,000 rows, int64 Zipf(1.1) keys over
1,000,000 ids, filter a>0, v=a*b+c, sum/count/mean/var), `highcard` (2,000,000,000
rows, int64 keys over 2^28 random ids, f32 LogNormal values, sum/count/mean: radix
partitioning by key hash on one GPU; with N GPUs the first pass routes every row to the
GPU owning its hash digit, one NCCL all-to-all, the owner runs the rest), `stress`
(200,000,000 rows, 10,000 groups, 1e9 + N(0,1e-3) with NaN / +-inf), `cpu-ref`
(1,000,000 rows, 1,000 groups), `stress-1k` and `bins` (1,000,000,000 f64 ticks in sorted
contiguous bins of 1..831 rows, mean 416: count/sum/sum_sq/min/max/first/last/mean/variance/std
per bin; its reference arm runs the reference's own CUDA kernel) and `pushdown` (1,000,000,000
rows, 256 int32 keys, a time-trending f64 price; `price > 190` over per-tile statistics built
once like a .tb header: skipped tiles are neither read on the device nor copied from the host).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload NAME]

Rank 0 prints one JSON line.  `value` is whole-job rows/s with the inputs resident
in HBM; `e2e` is the same metric through the public API with the step's inputs
copied from pinned host memory and the result read back inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "groupby-agg rows/s and HBM GB/s (frac of ~8 TB/s) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
KEY_SALT = 0x5EED5EED12345678

WORKLOADS = {
    "lowcard": dict(kind="dense", rows=1_000_000_000, groups=256, values=("uniform", -1.0, 1.0), nonfinite=None,
                    seed=0,
                    desc="low-cardinality sharded: 1,000,000,000 rows; int32 key uniform in [0,256); "
                         "f64 value ~U(-1,1); sum/count/min/max/mean/var; rows split evenly over the GPUs, "
                         "per-GPU state tables exchanged over NVLink peer memory and merged in rank order"),
    "cpu-ref": dict(kind="dense", rows=1_000_000, groups=1000, values=("normal", 0.0, 1.0), nonfinite=None, seed=0,
                    desc="1,000,000 rows; int32 key uniform in [0,1000); f64 value ~N(0,1); "
                         "sum/count/min/max/mean/var; seed 0"),
    "stress": dict(kind="dense", rows=200_000_000, groups=10000, values=("normal", 1e9, 1e-3),
                   nonfinite=(0.01, 0.001), seed=0,
                   desc="numerical stress: 200,000,000 rows; int32 key uniform in [0,10000); f64 value "
                        "1e9 + N(0,1e-3) with 1% NaN and 0.1% +-inf; count/sum/mean/var/min/max"),
    "stress-1k": dict(kind="dense", rows=200_000_000, groups=1000, values=("normal", 1e9, 1e-3),
                      nonfinite=(0.01, 0.001), seed=0,
                      desc="200,000,000 rows; int32 key uniform in [0,1000); f64 value 1e9 + N(0,1e-3), 1% NaN, "
                           "0.1% +-inf; count/mean/var/min/max"),
    "pipeline": dict(kind="pipeline", rows=100_000_000, ids=1_000_000, zipf=1.1, seed=0,
                     desc="fused pipeline: 100,000,000 rows; int64 key Zipf(1.1) over 1,000,000 random ids; "
                          "columns a,b,c f64 ~N(0,1); filter a>0, then v=a*b+c; sum/count/mean/var of v per key"),
    "bins": dict(kind="bins", rows=1_000_000_000, mean_bin=416, seed=0,
                 desc="segmented bin statistics: 1,000,000,000 f64 ticks ~N(100,1) in sorted contiguous bins of "
                      "1..831 rows (mean 416, about 2.4 M bins); count/sum/sum_sq/min/max/first/last/mean/"
                      "variance/std per bin"),
    "pushdown": dict(kind="pushdown", rows=1_000_000_000, groups=256, tile_rows=65536, threshold=190.0, seed=0,
                     desc="tile-skip pushdown: 1,000,000,000 rows; int32 key uniform in [0,256); f64 price = "
                          "100 + 100*row/rows + N(0,0.5) (time-ordered); filter price > 190 then "
                          "count/sum/mean/var of price per key; per-tile min/max statistics (65,536-row tiles) "
                          "built once outside the timed region, as a .tb file header holds them"),
    "highcard": dict(kind="highcard", rows=2_000_000_000, ids=1 << 28, seed=0,
                     desc="high-cardinality sharded: 2,000,000,000 rows; int64 key uniform over 2^28 random ids; "
                          "f32 value ~LogNormal(0,1); sum/count/mean; radix partitioning by key hash (with N GPUs "
                          "rows routed by hash digit, each GPU reads the rows of the digits it owns from the other "
                          "GPUs' buffers over NVLink peer memory and groups them)"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="lowcard", choices=sorted(WORKLOADS))
    ap.add_argument("--rows", type=int, default=None, help="override the workload's row count")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU work of the baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the parity check after the timed region")
    ap.add_argument("--ids", type=int, default=None, help="override the distinct-id count of a hash workload")
    ap.add_argument("--table-mode", default="auto", choices=["auto", "local", "direct", "bucket", "range", "sweep"],
                    help="global-table kernel: shared-memory pre-aggregation or direct atomics")
    ap.add_argument("--exchange", default="pull", choices=["pull", "nccl"],
                    help="multi-GPU high-cardinality exchange: owners read the senders' routed rows in place over "
                         "NVLink (pull), or NCCL all-to-all")
    return ap.parse_args()


# ---------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------

def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def traffic_model(workload: str):
    """DRAM bytes of the main kernel per row (+ fixed bytes per launch) from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None, None
    try:
        d = json.loads(p.read_text())[workload]
        return (float(d["dram_bytes_per_row"]), float(d.get("fixed_bytes_per_launch", 0.0))), d.get("source")
    except Exception:
        return None, None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        if self.uuid:
            cmd.insert(1, f"--id={self.uuid}")
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 10:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        smax = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower() == "active"})
        loaded = [x for x in sm if smax and x > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows)}




def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def zipf_table(wl):
    import oracle

    return oracle.zipf_cdf(wl["ids"], wl["zipf"])


def bin_boundaries(wl, n_rows):
    """Boundaries of the `bins` workload: bin sizes 1 + u, u uniform in [0, 2 * mean_bin - 1) from the
    workload's SplitMix64 stream, cut at n_rows (int64, n_bins + 1 entries)."""
    import numpy as np

    import oracle

    m = wl["mean_bin"]
    est = n_rows // m + n_rows // (4 * m) + 16
    sizes = oracle.gen_keys_uniform(est, 2 * m - 1, wl["seed"] + 7, 0).astype(np.int64) + 1
    b = np.concatenate([[0], np.cumsum(sizes)])
    b = b[b < n_rows]
    return np.append(b, n_rows).astype(np.int64)


def host_inputs(wl, start, count):
    """Rows [start, start+count) of the workload generated on the host (same recipes as the device
    generators; integer columns bit-identical)."""
    import oracle

    seed = wl["seed"]
    if wl["kind"] == "bins":
        return {"a": oracle.gen_values_normal(count, 100.0, 1.0, seed, start),
                "bounds": bin_boundaries(wl, start + count)}
    if wl["kind"] == "pushdown":
        import numpy as np

        total = wl.get("rows_total", wl["rows"])
        price = oracle.gen_values_normal(count, 0.0, 0.5, seed + 1, start) + (
            100.0 + 100.0 * (np.arange(start, start + count, dtype=np.float64) / total))
        return {"keys": oracle.gen_keys_uniform(count, wl["groups"], seed, start), "a": price}
    if wl["kind"] == "dense":
        keys = oracle.gen_keys_uniform(count, wl["groups"], seed, start)
        kind, a, b = wl["values"]
        if kind == "uniform":
            vals = oracle.gen_values_uniform(count, a, b, seed, start)
        else:
            vals = oracle.gen_values_normal(count, a, b, seed, start)
        if wl["nonfinite"]:
            vals = oracle.inject_nonfinite(vals, wl["nonfinite"][0], wl["nonfinite"][1], seed, start)
        return {"keys": keys, "a": vals}
    if wl["kind"] == "pipeline":
        return {"keys": oracle.gen_keys_cdf(count, zipf_table(wl), KEY_SALT, seed, start),
                "a": oracle.gen_values_normal(count, 0.0, 1.0, seed + 1, start),
                "b": oracle.gen_values_normal(count, 0.0, 1.0, seed + 2, start),
                "c": oracle.gen_values_normal(count, 0.0, 1.0, seed + 3, start)}
    return {"keys": oracle.gen_keys_ids(count, wl["ids"], KEY_SALT, seed, start),
            "a": oracle.gen_values_lognormal_f32(count, 0.0, 1.0, seed, start)}


def cpu_groupby(wl, cols, threads):
    """The reference's CPU groupby (oracle port) over host columns, on `threads` threads."""
    import numpy as np

    import oracle

    if wl["kind"] == "dense":
        return oracle.moments_grouped_mt(cols["a"], cols["keys"], wl["groups"], threads=threads)
    if wl["kind"] == "pushdown":
        mask = oracle.filter_mask("gt", wl["threshold"], cols["a"])
        return oracle.moments_grouped_mt(cols["a"], cols["keys"], wl["groups"], threads=threads, mask=mask)
    if wl["kind"] == "bins":
        # contiguous bin ranges per thread (the C oracle runs without the GIL)
        b, d = cols["bounds"], cols["a"]
        nb = b.size - 1
        cuts = [nb * t // threads for t in range(threads + 1)]
        res = [None] * threads

        def bwork(t):
            lo, hi = cuts[t], cuts[t + 1]
            res[t] = oracle.bin_stats(d, b[lo:hi + 1])

        ths = [threading.Thread(target=bwork, args=(t,)) for t in range(threads)]
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        return res
    keys = cols["keys"]
    if wl["kind"] == "pipeline":
        mask = oracle.filter_mask("gt", 0.0, cols["a"])
        v = oracle.map2("a + b", oracle.map2("a * b", cols["a"], cols["b"]), cols["c"])
        live = ((mask[np.arange(keys.size) // 64] >> (np.arange(keys.size) % 64).astype(np.uint64))
                & np.uint64(1)).astype(bool)
        keys, v = keys[live], v[live]
    else:
        v = cols["a"].astype(np.float64)
    if threads <= 1:
        return oracle.groupby_i64(keys, v)
    # key-disjoint buckets, one per thread (the C oracle runs without the GIL)
    bucket = (keys.view(np.uint64) * np.uint64(0x9E3779B97F4A7C15)) >> np.uint64(58)
    bucket = (bucket % np.uint64(threads)).astype(np.int64)
    order = np.argsort(bucket, kind="stable")
    bounds = np.searchsorted(bucket[order], np.arange(threads + 1))
    res = [None] * threads

    def work(t):
        idx = order[bounds[t]:bounds[t + 1]]
        res[t] = oracle.groupby_i64(keys[idx], v[idx])

    ths = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    return res


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def single_thread_baseline(wl, n_rows, target_s=6.0):
    """The reference's own execution model: its CPU path is single-threaded
    (compute_engine.rs:229-230), so the oracle port on one thread over a bounded prefix."""
    sample = cpu_sample_rows(wl, target_s, 1, n_rows)
    cols = host_inputs(wl, 0, sample)
    t0 = time.perf_counter()
    cpu_groupby(wl, cols, 1)
    dt = time.perf_counter() - t0
    return {"value": sample / dt, "unit": "rows/s", "cores": 1, "kind": "port",
            "sample": f"first {sample} rows of the workload on one thread",
            "cpu_model": cpu_model(), "nproc": os.cpu_count()}


def cpu_sample_rows(wl, target_s, threads, n_rows):
    """Rows the oracle processes in about target_s seconds on `threads` threads (calibrated)."""
    n0 = min(2_000_000, n_rows)
    cols = host_inputs(wl, 0, n0)
    t0 = time.perf_counter()
    cpu_groupby(wl, cols, threads)
    rate = n0 / (time.perf_counter() - t0)
    return min(max(n0, int(rate * target_s)), n_rows, 200_000_000)


def bytes_per_row(wl) -> int:
    """Algorithmic input bytes per row: every column read once."""
    return {"dense": 12, "pipeline": 32, "highcard": 12, "bins": 8, "pushdown": 12}[wl["kind"]]


def base_line(args, wl, n_rows, world):
    bpr = bytes_per_row(wl)
    cfg = {"workload": wl["desc"], "rows": n_rows, "bytes_per_row": bpr, "parallelism": f"row-shards x{world}",
           "l2": "inputs far larger than the 126 MB L2; no flush needed between steps"
           if n_rows * bpr > 1 << 30 else "inputs smaller than L2: L2 flushed between steps"}
    if "groups" in wl:
        cfg["n_groups"] = wl["groups"]
    elif "ids" in wl:
        cfg["distinct_ids"] = wl["ids"]
    else:
        cfg["mean_bin_rows"] = wl["mean_bin"]
    if args.table_mode != "auto":
        cfg["table_mode"] = args.table_mode
    return {
        "metric": METRIC,
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic (counter-based SplitMix64 streams, same shapes and distributions as the configuration)",
        "config": cfg,
    }


# ---------------------------------------------------------------------------------
# the reference arm: the reference's CPU groupby (oracle port) on the host cores
# ---------------------------------------------------------------------------------

def run_reference_bins(args, wl, n_rows, world):
    """The reference's own bin-statistics CUDA kernel (src/winrapids/kernels/bin_stats.cu, built
    from its source into oracle/_ref) on this GPU: the reference has no CPU path for this row."""
    import ctypes as C

    import numpy as np
    import torch

    lib_path = ROOT / "oracle" / "_ref" / "libref_bin_stats.so"
    line = base_line(args, wl, n_rows, world)
    if not lib_path.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_bin_stats.so was not built "
                                                                "(the reference tree was absent at build time)"}))
        return
    L = C.CDLL(str(lib_path))
    dev = torch.device("cuda:0")
    import winrapids_b200 as wb

    ctx = wb.Context(0)
    data = torch.empty(n_rows, dtype=torch.float64, device=dev)
    ctx.gen_values_normal(data, 100.0, 1.0, wl["seed"], 0)
    bnd = torch.as_tensor(bin_boundaries(wl, n_rows)).to(dev)
    nb = int(bnd.numel()) - 1
    outs = [torch.empty(nb, dtype=torch.float64, device=dev) for _ in range(6)]
    cnt = torch.empty(nb, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    args_c = [C.c_void_p(data.data_ptr()), C.c_void_p(bnd.data_ptr())] + [C.c_void_p(o.data_ptr()) for o in outs]
    args_c += [C.c_void_p(cnt.data_ptr()), C.c_int(nb), C.c_void_p(stream.cuda_stream)]

    def step():
        assert L.ref_fused_bin_stats(*args_c) == 0

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    value = n_rows * args.steps / (ms / 1e3)
    line.update({
        "impl": "reference",
        "value": value,
        "ms_per_step": ms / args.steps,
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": 0, "kind": "reference",
                         "sample": "the whole workload per step on the GPU: the reference's fused_bin_stats "
                                   "kernel (one thread per bin), built from its source"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "device": ctx.name,
    })
    print(json.dumps(line), flush=True)


def run_reference(args, wl, n_rows, world, rank):
    if rank != 0:
        return
    if wl["kind"] == "bins":
        run_reference_bins(args, wl, n_rows, world)
        return
    threads = cpu_threads()
    per_step_s = max(2.0, min(20.0, 150.0 / max(1, args.steps + args.warmup)))
    sample = cpu_sample_rows(wl, per_step_s, threads, n_rows)
    cols = host_inputs(wl, 0, sample)
    for _ in range(args.warmup):
        cpu_groupby(wl, cols, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_groupby(wl, cols, threads)
    dt = time.perf_counter() - t0
    value = sample * args.steps / dt
    line = base_line(args, wl, n_rows, world)
    how = {"dense": "exact Kulisch groupby, per-thread registers merged in row-range order",
           "pushdown": "filter mask, then exact Kulisch groupby of the passing rows (no tile skipping)",
           "bins": "serial per-bin loop of the reference kernel, contiguous bin ranges per thread"}.get(
        wl["kind"], "sort-based exact groupby of int64 keys, key-disjoint buckets per thread")
    line.update({
        "impl": "reference",
        "value": value,
        "ms_per_step": dt * 1000.0 / args.steps,
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"first {sample} rows of the workload per step ({how})"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })
    line["cpu_baseline"]["cpu_model"] = cpu_model()
    line["cpu_baseline"]["nproc"] = os.cpu_count()
    if wl["kind"] != "bins":
        line["cpu_baseline"]["single_thread"] = single_thread_baseline(wl, n_rows)
    if wl["kind"] == "dense" and world == 1:
        line["reference_gpu"] = reference_gpu_scatter(args, wl, n_rows)
    print(json.dumps(line), flush=True)


def reference_gpu_scatter(args, wl, n_rows):
    """The reference's own best GPU groupby kernels (scatter_stats_smem / scatter_stats_warp of
    crates/tambear/src/hash_scatter.rs, built from its source into oracle/_ref) timed on this GPU
    over the same workload: they compute sum, sum of squares and count per group (no min / max,
    no NaN handling), one row per thread, with the reference's launch configuration."""
    import ctypes as C

    try:
        import torch
    except Exception as exc:  # pragma: no cover
        return {"unavailable": f"torch: {exc}"}
    lib_path = ROOT / "oracle" / "_ref" / "libref_hash_scatter.so"
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    if not lib_path.exists():
        return {"unavailable": "oracle/_ref/libref_hash_scatter.so was not built"}
    if n_rows >= 1 << 31:
        return {"unavailable": "the reference kernels take an int row count (< 2^31)"}
    import winrapids_b200 as wb

    L = C.CDLL(str(lib_path))
    ctx = wb.Context(0)  # input generation only (the workload's SplitMix64 recipe)
    G = wl["groups"]
    dk = torch.empty(n_rows, dtype=torch.int32, device="cuda:0")
    dv = torch.empty(n_rows, dtype=torch.float64, device="cuda:0")
    ctx.gen_keys_uniform(dk, G, wl["seed"], 0)
    kind, a, b = wl["values"]
    (ctx.gen_values_uniform if kind == "uniform" else ctx.gen_values_normal)(dv, a, b, wl["seed"], 0)
    if wl["nonfinite"]:
        ctx.gen_inject_nonfinite(dv, wl["nonfinite"][0], wl["nonfinite"][1], wl["seed"], 0)
    outs = [torch.empty(G, dtype=torch.float64, device="cuda:0") for _ in range(3)]
    stream = torch.cuda.current_stream()
    peak, peak_kind = measured_peak()
    res = {"config": "same rows as the workload; outputs sum / sum_sq / count only", "kernels": {}}
    for kid, name in ((1, "scatter_stats_smem"), (2, "scatter_stats_warp")):
        argv = [C.c_int(kid), C.c_void_p(dk.data_ptr()), C.c_void_p(dv.data_ptr())]
        argv += [C.c_void_p(o.data_ptr()) for o in outs]
        argv += [C.c_longlong(n_rows), C.c_int(G), C.c_void_p(stream.cuda_stream)]
        if L.ref_scatter_stats(*argv) != 0:
            res["kernels"][name] = {"unavailable": "launch failed (shared memory beyond the limit?)"}
            continue
        torch.cuda.synchronize()
        steps = max(3, min(args.steps, 10))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            L.ref_scatter_stats(*argv)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        gbs = n_rows * 12 / (ms / 1e3) / 1e9
        res["kernels"][name] = {"ms_per_step": ms, "rows_per_s": n_rows / (ms / 1e3), "hbm_gbs": gbs,
                                "frac": gbs / peak, "peak": peak, "peak_source": peak_kind}
    ctx.close()
    return res


# ---------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------

def dense_kernel_name(G: int, mode: str) -> str:
    """Main kernel of a plain dense groupby (count/sum/min/max/mean/var) under a table mode."""
    if G <= 512 or (mode != "auto" and G <= 1024):
        return "dense_moments_kernel"
    if mode == "auto" and (227 * 1024 // G - 60) // 8 >= 4:  # rank and sweep: one range, four columns
        return "sweep_table_kernel"
    if mode == "sweep":  # up to 8 ranges with two value columns a group
        for r in range(1, 9):
            gr = -(-G // r)
            if (227 * 1024 // gr - 60) // 8 >= 2:
                return "sweep_table_kernel"
    if mode in ("auto", "range", "sweep") and -(-G // (225 * 1024 // 56)) <= 8:
        return "range_table_kernel"
    return "table_kernel"


class DenseJob:
    """int32 keys in [0, G): the shared-memory column kernel (G <= 1024) or the global table."""

    def __init__(self, ctx, wl, lo, hi, world, dist, dev):
        import torch

        self.ctx, self.wl, self.lo, self.world, self.dist = ctx, wl, lo, world, dist
        G = self.G = wl["groups"]
        n = self.n_local = hi - lo
        self.kernel = dense_kernel_name(G, wl.get("table_mode", "auto"))
        self.bpr = 12
        dk = torch.empty(n, dtype=torch.int32, device=dev)
        dv = torch.empty(n, dtype=torch.float64, device=dev)
        seed = wl["seed"]
        ctx.gen_keys_uniform(dk, G, seed, lo)
        kind, a, b = wl["values"]
        if kind == "uniform":
            ctx.gen_values_uniform(dv, a, b, seed, lo)
        else:
            ctx.gen_values_normal(dv, a, b, seed, lo)
        if wl["nonfinite"]:
            ctx.gen_inject_nonfinite(dv, wl["nonfinite"][0], wl["nonfinite"][1], seed, lo)
        self.inputs = [dk, dv]
        self.out = ctx.alloc_moments(G)
        self.sharded = None
        self.exchange = None
        if world > 1:
            from winrapids_b200.sharded import PeerMappingError, PeerShardedDenseGroupby, ShardedDenseGroupby

            rank = int(os.environ.get("RANK", "0"))
            try:  # the exchange over NVLink peer memory; the NCCL all-gather if the mapping fails
                self.sharded = PeerShardedDenseGroupby(ctx, dist, world, rank, G, self.out, dev)
                self.exchange = "peer memory (state tables stored into every rank's buffer over NVLink)"
            except PeerMappingError as exc:
                self.sharded = ShardedDenseGroupby(ctx, dist, world, G, self.out, dev)
                self.exchange = f"NCCL all-gather ({exc})"

    def step(self, inputs):
        keys, vals = inputs
        if self.sharded is None:
            self.ctx.groupby_dense(keys, vals, self.G, out=self.out, sync=False)
        else:
            self.sharded.step(keys, vals, self.lo)

    def kernel_bytes(self) -> int:
        return self.n_local * self.bpr

    def check(self, dev_in, dist, world):
        return dense_check(dev_in[0], dev_in[1], self.out, self.G, dist)

    def read_result(self, host: dict) -> int:
        import torch

        for f, t in self.out.items():
            if f not in host:
                host[f] = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
            host[f].copy_(t, non_blocking=True)
        return sum(t.numel() * 8 for t in self.out.values())


class HashJob:
    """int64 keys through the hash table: `pipeline` (filter + expression, Zipf keys) and `highcard`
    (f32 values, sum/count/mean; owner-sharded when world > 1: rows routed by hash digit and stored
    into the owners' buffers over NVLink peer memory)."""

    def __init__(self, ctx, wl, lo, hi, world, dist, dev):
        import torch

        import winrapids_b200 as wb

        self.ctx, self.wl, self.world, self.dist = ctx, wl, world, dist
        n = self.n_local = hi - lo
        radix = (wl["kind"] == "highcard" and wl.get("table_mode", "auto") in ("auto", "radix")
                 and (world > 1 or (n >= 1 << 24 and (1 << 22) <= wl["ids"] <= (1 << 28))))
        # the pipeline's outputs carry no extrema: its rows take the per-warp queued shared table
        self.kernel = ("rx_scatter_kernel + rx_agg_kernel (radix passes)" if radix else
                       "table_queue_kernel" if wl["kind"] == "pipeline" else "table_kernel")
        seed = wl["seed"]
        keys = torch.empty(n, dtype=torch.int64, device=dev)
        if wl["kind"] == "pipeline":
            self.bpr = 32
            self.fields = ("count", "sum", "mean", "m2", "var_pop", "var_samp")
            cdf = torch.as_tensor(zipf_table(wl)).to(dev)
            ctx.gen_keys_cdf(keys, cdf, KEY_SALT, seed, lo)
            cols = []
            for j in (1, 2, 3):
                t = torch.empty(n, dtype=torch.float64, device=dev)
                ctx.gen_values_normal(t, 0.0, 1.0, seed + j, lo)
                cols.append(t)
            self.inputs = [keys] + cols
            self.op = dict(expr="a*b+c", pred=">", threshold=0.0)
        else:
            self.bpr = 12
            self.fields = wb.SUMCOUNT_FIELDS
            ctx.gen_keys_ids(keys, wl["ids"], KEY_SALT, seed, lo)
            vals = torch.empty(n, dtype=torch.float32, device=dev)
            ctx.gen_values_lognormal_f32(vals, 0.0, 1.0, seed, lo)
            self.inputs = [keys, vals]
            self.op = {}
        ids = wl["ids"]
        if world == 1:
            self.max_groups = ids
            self.out_keys = torch.empty(ids, dtype=torch.int64, device=dev)
            self.out = {f: torch.empty(ids, dtype=torch.float64, device=dev) for f in self.fields}
            self.ng = torch.zeros(1, dtype=torch.int64, device=dev)
            self.sharded = None
        else:
            from winrapids_b200.sharded import PeerMappingError, ShardedHashGroupby

            per_owner = int(ids / world * 1.05) + 4096
            how = wl.get("exchange", "pull") if radix else "nccl"
            try:
                self.sharded = ShardedHashGroupby(ctx, dist, world, n, per_owner, self.fields, dev, exchange=how)
                self.exchange = {"pull": "peer memory (owners read the senders' routed rows in place over NVLink)",
                                 "nccl": "NCCL all-to-all of the routed rows"}[how]
            except PeerMappingError as exc:
                self.sharded = ShardedHashGroupby(ctx, dist, world, n, per_owner, self.fields, dev)
                self.exchange = f"NCCL all-to-all ({exc})"
            self.out_keys, self.out, self.ng = self.sharded.out_keys, self.sharded.out, self.sharded.n_groups

    def _cols(self, inputs):
        keys, a = inputs[0], inputs[1]
        b = inputs[2] if len(inputs) > 2 else None
        c = inputs[3] if len(inputs) > 3 else None
        return keys, a, b, c

    def step(self, inputs):
        keys, a, b, c = self._cols(inputs)
        if self.sharded is None:
            self.ctx.groupby_hash_into(keys, a, self.max_groups, self.out_keys, self.out, self.ng, b=b, c=c,
                                       **self.op)
        else:
            self.sharded.step(keys, a, b=b, c=c, **self.op)

    def check(self, dev_in, dist, world):
        return hash_check(self, dev_in, dist, world)

    def extra(self, args) -> dict:
        """Whether the last timed step's radix passes fell back to the global table (0: no)."""
        if "rx_" not in self.kernel:
            return {}
        return {"radix_fallback": self.ctx.radix_fallback()}

    def kernel_bytes(self) -> int:
        # the shard's columns (one GPU) or the received rows (hash and value, or key and f64 value)
        return self.n_local * self.bpr if self.sharded is None else self.sharded.n_recv * self.sharded.recv_bytes_per_row

    def read_result(self, host: dict) -> int:
        import torch

        g = int(self.ng.item())  # the group count decides how much to read back
        total = 8
        for f, t in [("keys", self.out_keys)] + list(self.out.items()):
            if f not in host:
                host[f] = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
            host[f][:g].copy_(t[:g], non_blocking=True)
            total += g * 8
        return total


class PushdownJob:
    """Filter + groupby with tile skipping: the skip mask from per-tile statistics, the row mask of
    the surviving tiles, then the fused filter + groupby, which reads no column of a masked-out row."""

    def __init__(self, ctx, wl, lo, hi, world, dist, dev):
        import torch

        self.ctx, self.wl = ctx, wl
        self.kernel = "dense_moments_kernel"
        self.bpr = 12
        self.G = wl["groups"]
        self.tile_rows = wl["tile_rows"]
        self.thr = wl["threshold"]
        n = self.n_local = hi - lo
        total = wl["rows_total"]
        keys = torch.empty(n, dtype=torch.int32, device=dev)
        ctx.gen_keys_uniform(keys, self.G, wl["seed"], lo)
        price = torch.empty(n, dtype=torch.float64, device=dev)
        ctx.gen_values_normal(price, 0.0, 0.5, wl["seed"] + 1, lo)
        price += 100.0 + 100.0 * (torch.arange(lo, hi, dtype=torch.float64, device=dev) / total)
        self.inputs = [keys, price]
        self.stats = ctx.tile_stats(price, self.tile_rows)  # the header: built once, outside the timed region
        self.n_tiles = int(self.stats.shape[0])
        self.mask = torch.empty((n + 63) // 64, dtype=torch.int64, device=dev)
        self.out = ctx.alloc_moments(self.G, ("count", "sum", "mean", "m2", "var_pop", "var_samp"))
        skip = ctx.tile_skip_mask(self.stats, ">", self.thr).cpu().numpy()
        self.live_tiles = int((skip == 0).sum())
        self.live_rows = sum(min(self.tile_rows, n - t * self.tile_rows) for t in range(self.n_tiles) if not skip[t])

    def step(self, inputs):
        keys, price = inputs
        skip = self.ctx.tile_skip_mask(self.stats, ">", self.thr)
        self.ctx.mask_skip_tiles(skip, self.tile_rows, self.n_local, out=self.mask)
        self.ctx.groupby_dense_columns(keys, price, self.G, pred=">", threshold=self.thr, mask=self.mask,
                                       out=self.out, sync=False)

    def kernel_bytes(self) -> int:
        # the table kernel reads the row mask and the key and price of the rows of surviving tiles
        return self.n_local // 8 + self.live_rows * 12

    def e2e_copy(self, dev_in, host_in) -> int:
        """Host -> device only for the runs of tiles the skip mask keeps (the skip flags come back
        from the device first, n_tiles bytes)."""
        skip = self.ctx.tile_skip_mask(self.stats, ">", self.thr).cpu().numpy()
        total, t, tr, n = 0, 0, self.tile_rows, self.n_local
        while t < self.n_tiles:
            if skip[t]:
                t += 1
                continue
            u = t
            while u < self.n_tiles and not skip[u]:
                u += 1
            r0, r1 = t * tr, min(u * tr, n)
            for d, h in zip(dev_in, host_in):
                d[r0:r1].copy_(h[r0:r1], non_blocking=True)
                total += (r1 - r0) * h.element_size()
            t = u
        return total + self.n_tiles

    def extra(self, args) -> dict:
        """The same query without tile skipping (every row's price read and compared)."""
        import torch

        keys, price = self.inputs
        for _ in range(2):
            self.ctx.groupby_dense_columns(keys, price, self.G, pred=">", threshold=self.thr, out=self.out, sync=False)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k = max(3, min(args.steps, 10))
        e0.record()
        for _ in range(k):
            self.ctx.groupby_dense_columns(keys, price, self.G, pred=">", threshold=self.thr, out=self.out, sync=False)
        e1.record()
        torch.cuda.synchronize()
        self.ctx.sync()
        return {"pushdown": {"tiles": self.n_tiles, "tiles_read": self.live_tiles, "rows_read": self.live_rows,
                             "ms_per_step_without_skipping": e0.elapsed_time(e1) / k}}

    def read_result(self, host: dict) -> int:
        import torch

        for f, t in self.out.items():
            if f not in host:
                host[f] = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
            host[f].copy_(t, non_blocking=True)
        return sum(t.numel() * 8 for t in self.out.values())


class BinsJob:
    """Sorted contiguous bins (tbgb_fused_bin_stats).  With N GPUs each takes a contiguous range of
    bins and the rows they cover (no exchange: bins are independent)."""

    def __init__(self, ctx, wl, lo, hi, world, dist, dev, rank=0):
        import numpy as np
        import torch

        import winrapids_b200 as wb

        self.ctx = ctx
        self.kernel = "bin_chunk_kernel"
        self.bpr = 8
        n = wl["rows_total"]
        b = bin_boundaries(wl, n)
        nb = b.size - 1
        b0, b1 = nb * rank // world, nb * (rank + 1) // world
        r0, r1 = int(b[b0]), int(b[b1])
        self.n_local = r1 - r0
        self.nb = b1 - b0
        data = torch.empty(self.n_local, dtype=torch.float64, device=dev)
        ctx.gen_values_normal(data, 100.0, 1.0, wl["seed"], r0)
        bnd = torch.as_tensor(np.ascontiguousarray(b[b0:b1 + 1] - r0)).to(dev)
        self.inputs = [data, bnd]
        self.out = {f: torch.empty(self.nb, dtype=torch.int32 if f == "count" else torch.float64, device=dev)
                    for f in wb._lib.BIN_STATS_FIELDS}

    def step(self, inputs):
        self.ctx.fused_bin_stats(inputs[0], inputs[1], out=self.out, sync=False)

    def kernel_bytes(self) -> int:
        # ticks read once, boundaries read, 9 f64 + 1 int32 outputs written per bin
        return self.n_local * 8 + (self.nb + 1) * 8 + self.nb * 76

    def read_result(self, host: dict) -> int:
        import torch

        total = 0
        for f, t in self.out.items():
            if f not in host:
                host[f] = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
            host[f].copy_(t, non_blocking=True)
            total += t.numel() * t.element_size()
        return total


# ---------------------------------------------------------------------------------
# parity check after the timed region (every N): the merged result against torch
# reductions of the same device inputs, all-reduced over the ranks
# ---------------------------------------------------------------------------------

SUM_TOL = 1e-12   # |sum - want| <= 1e-12 * sum |x| over the group's finite values
VAR_RTOL = 1e-9   # m2 / variances relative
CHUNK_ROWS = 1 << 22


def _allreduce(dist, t, op):
    if dist is not None:
        dist.all_reduce(t, op=op)
    return t


def _chunked_index(keys_long, G):
    """Row -> chunk * G + key, so that per-(chunk, group) partials see few rows each
    (few atomics on one address, and short f64 sums)."""
    import torch

    n = keys_long.numel()
    chunk = torch.arange(n, device=keys_long.device, dtype=torch.int64) // CHUNK_ROWS
    return chunk * G + keys_long, (n + CHUNK_ROWS - 1) // CHUNK_ROWS


def dense_check(keys, vals, out, G, dist):
    """Counts bit-exact, min/max bit-exact (a zero is compared by value: torch's reduction does not
    order +-0 ties), sums within 1e-12 * sum|x|, mean consistent, m2 / variances within 1e-9
    relative, against chunked torch reductions of this rank's rows all-reduced over the ranks."""
    import torch

    RO = dist.ReduceOp if dist is not None else None
    dev = vals.device
    k = keys.long()
    if keys.numel() and (int(k.min()) < 0 or int(k.max()) >= G):
        return {"ok": False, "why": "key outside [0, G)"}
    idx, nch = _chunked_index(k, G)
    nan = torch.isnan(vals)
    fin = torch.isfinite(vals)
    zero = torch.zeros((), dtype=torch.float64, device=dev)

    def gsum(w):
        t = torch.zeros(nch * G, dtype=torch.float64, device=dev).index_add_(0, idx, w)
        return t.view(nch, G).sum(0)

    cnt = gsum((~nan).double())
    nf = gsum(fin.double())
    s = gsum(torch.where(fin, vals, zero))
    absum = gsum(torch.where(fin, vals.abs(), zero))
    inf = torch.tensor(float("inf"), dtype=torch.float64, device=dev)
    mn = torch.full((nch * G,), float("inf"), dtype=torch.float64, device=dev).scatter_reduce_(
        0, idx, torch.where(nan, inf, vals), "amin").view(nch, G).amin(0)
    mx = torch.full((nch * G,), float("-inf"), dtype=torch.float64, device=dev).scatter_reduce_(
        0, idx, torch.where(nan, -inf, vals), "amax").view(nch, G).amax(0)
    K = torch.full((nch * G,), float("inf"), dtype=torch.float64, device=dev).scatter_reduce_(
        0, idx, torch.where(fin, vals, inf), "amin").view(nch, G).amin(0)
    sums = torch.stack([cnt, nf, s, absum])
    _allreduce(dist, sums, RO.SUM if RO else None)
    _allreduce(dist, mn, RO.MIN if RO else None)
    _allreduce(dist, mx, RO.MAX if RO else None)
    _allreduce(dist, K, RO.MIN if RO else None)
    cnt, nf, s, absum = sums
    K = torch.where(torch.isfinite(K), K, zero)
    # m2 = sum over finite v of (v - mean)^2, mean = sum / count; shifted by K so the sums stay exact
    d = torch.where(fin, vals - K[k], zero)
    S1 = gsum(d)
    _allreduce(dist, S1, RO.SUM if RO else None)
    c1 = torch.where(cnt > 0, cnt, torch.ones_like(cnt))
    c = torch.where(cnt > 0, S1 / c1 + K * (nf / c1 - 1.0), zero)  # mean - K
    m2 = gsum(torch.where(fin, (d - c[k]) ** 2, zero))
    _allreduce(dist, m2, RO.SUM if RO else None)

    got = {f: t.double() for f, t in out.items()}
    res = {}
    res["count"] = bool(torch.equal(got["count"], cnt))
    for f, w in (("min", mn), ("max", mx)):
        g = got[f]
        same_bits = g.view(torch.int64) == w.view(torch.int64)
        res[f] = bool(torch.all(same_bits | ((w == 0) & (g == 0))))
    res["sum"] = bool(torch.all((got["sum"] - s).abs() <= SUM_TOL * absum))
    mean_w = torch.where(cnt > 0, s / c1, torch.full_like(s, float("nan")))
    res["mean"] = bool(torch.all(torch.where(cnt > 0, (got["mean"] - mean_w).abs() <= SUM_TOL * absum / c1 + 1e-300,
                                             torch.isnan(got["mean"]))))
    worst = 0.0
    for f, w in (("m2", torch.where(cnt > 0, m2, zero)),
                 ("var_pop", torch.where(cnt > 0, m2 / c1, torch.full_like(m2, float("nan")))),
                 ("var_samp", torch.where(cnt > 1, m2 / (cnt - 1).clamp(min=1), torch.full_like(m2, float("nan"))))):
        if f not in got:
            continue
        g = got[f]
        nanw = torch.isnan(w)
        okf = torch.equal(torch.isnan(g), nanw)
        rel = ((g - w).abs() / w.abs().clamp(min=1e-300))[~nanw & (w != 0)]
        worst = max(worst, float(rel.max()) if rel.numel() else 0.0)
        okf = okf and bool(torch.all(torch.where(nanw, True, (g - w).abs() <= VAR_RTOL * w.abs())))
        res[f] = okf
    return {"ok": all(res.values()), "fields": res, "worst_var_rel": worst, "groups": G,
            "method": "chunked torch reductions of the same device inputs, all-reduced over ranks"}


def _fingerprint_bucket(keys, bits):
    """A bucket of 2^bits per int64 key (multiplicative hash; independent of the library's)."""
    import torch

    h = keys * -7046029254386353131  # 0x9E3779B97F4A7C15 as a signed int64 (wrapping product)
    return (h >> (64 - bits)) & ((1 << bits) - 1)


def _globally_unique(keys, dist, world, dev):
    """No key appears twice in the union of the ranks' key lists (keys routed by a hash of their
    own to a checking rank, then sorted there)."""
    import torch

    if dist is None or world == 1:
        sk = torch.sort(keys).values
        return bool(sk.numel() < 2 or torch.all(sk[1:] != sk[:-1]))
    dest = _fingerprint_bucket(keys, 20) % world
    order = torch.argsort(dest)
    send = keys[order]
    sc = torch.bincount(dest, minlength=world)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc)
    recv = torch.empty(int(rc.sum()), dtype=torch.int64, device=dev)
    dist.all_to_all_single(recv, send, output_split_sizes=rc.tolist(), input_split_sizes=sc.tolist())
    sk = torch.sort(recv).values
    return bool(sk.numel() < 2 or torch.all(sk[1:] != sk[:-1]))


def hash_check(job, dev_in, dist, world):
    """int64 keys.  Every rank: its result groups' keys are unique across all ranks; per bucket of
    2^24 key hashes, the result's counts equal the input's (exact) and its sums are within
    1e-12 * sum|x| of the input's (all-reduced over ranks); mean = sum / count.  With one rank,
    additionally every group's count, sum and (when present) m2 against torch reductions over the
    rows mapped to their group by a sorted search.  Rows are visited in chunks to bound memory."""
    import torch

    RO = dist.ReduceOp if dist is not None else None
    dev = dev_in[0].device
    n = dev_in[0].numel()
    step = 1 << 27

    def rows(lo, hi):
        """(keys, v) of rows [lo, hi) that take part, v in f64."""
        keys = dev_in[0][lo:hi]
        a = dev_in[1][lo:hi].double()
        if len(dev_in) > 2:  # the fused pipeline: a > 0 (NaN fails), v = (a * b) + c with two roundings
            live = a > job.op["threshold"]
            prod = a * dev_in[2][lo:hi]
            v = prod + dev_in[3][lo:hi]
            return keys[live], v[live]
        return keys, a

    g = int(job.ng.item())
    rk = job.out_keys[:g]
    got = {f: t[:g] for f, t in job.out.items()}
    res = {"unique": _globally_unique(rk, dist, world, dev)}
    bits = 24
    nb = 1 << bits
    zero = torch.zeros((), dtype=torch.float64, device=dev)
    want = torch.zeros(3, nb, dtype=torch.float64, device=dev)
    for lo in range(0, n, step):
        keys, v = rows(lo, min(n, lo + step))
        fin = torch.isfinite(v)
        bi = _fingerprint_bucket(keys, bits)
        want[0].index_add_(0, bi, (~torch.isnan(v)).double())
        want[1].index_add_(0, bi, torch.where(fin, v, zero))
        want[2].index_add_(0, bi, torch.where(fin, v.abs(), zero))
        del keys, v, fin, bi
    br = _fingerprint_bucket(rk, bits)
    have = torch.stack([torch.zeros(nb, dtype=torch.float64, device=dev).index_add_(0, br, got[f])
                        for f in ("count", "sum")])
    _allreduce(dist, want, RO.SUM if RO else None)
    _allreduce(dist, have, RO.SUM if RO else None)
    res["bucket_counts"] = bool(torch.equal(have[0], want[0]))
    res["bucket_sums"] = bool(torch.all((have[1] - want[1]).abs() <= SUM_TOL * want[2] + 1e-300))
    del want, have, br
    c = got["count"]
    c1 = torch.where(c > 0, c, torch.ones_like(c))
    mean_w = torch.where(c > 0, got["sum"] / c1, torch.full_like(c, float("nan")))
    res["mean"] = bool(torch.all(torch.where(c > 0, (got["mean"] - mean_w).abs() <= 1e-15 * mean_w.abs(),
                                             torch.isnan(got["mean"]))))
    if world == 1 and g > 0:
        sk, perm = torch.sort(rk)
        cnt = torch.zeros(g, dtype=torch.float64, device=dev)
        s = torch.zeros(g, dtype=torch.float64, device=dev)
        absum = torch.zeros(g, dtype=torch.float64, device=dev)
        found = True
        for lo in range(0, n, step):
            keys, v = rows(lo, min(n, lo + step))
            pos = torch.searchsorted(sk, keys).clamp(max=g - 1)
            found = found and bool(torch.equal(sk[pos], keys))
            gi = perm[pos]
            fin = torch.isfinite(v)
            cnt.index_add_(0, gi, (~torch.isnan(v)).double())
            s.index_add_(0, gi, torch.where(fin, v, zero))
            absum.index_add_(0, gi, torch.where(fin, v.abs(), zero))
            del keys, v, pos, gi, fin
        res["every_row_has_its_group"] = found
        res["count"] = bool(torch.equal(c, cnt))
        res["sum"] = bool(torch.all((got["sum"] - s).abs() <= SUM_TOL * absum))
        if "m2" in got:
            mu = torch.where(cnt > 0, s / torch.where(cnt > 0, cnt, torch.ones_like(cnt)), zero)
            m2 = torch.zeros(g, dtype=torch.float64, device=dev)
            for lo in range(0, n, step):
                keys, v = rows(lo, min(n, lo + step))
                gi = perm[torch.searchsorted(sk, keys).clamp(max=g - 1)]
                m2.index_add_(0, gi, torch.where(torch.isfinite(v), (v - mu[gi]) ** 2, zero))
                del keys, v, gi
            res["m2"] = bool(torch.all((got["m2"] - m2).abs() <= VAR_RTOL * m2.abs() + 1e-300))
    ok = torch.tensor([1.0 if all(res.values()) else 0.0], device=dev)
    _allreduce(dist, ok, RO.MIN if RO else None)
    return {"ok": bool(ok.item() == 1.0), "fields": res, "groups_this_rank": g,
            "method": "global key uniqueness, per-bucket count/sum fingerprints over 2^24 key hashes"
                      + ("; per-group count/sum/m2 by sorted search" if world == 1 else "")}


def run_ours(args, wl, n_rows, world, rank, local_rank, dist):
    import torch

    import winrapids_b200 as wb

    dev = torch.device(f"cuda:{local_rank}")
    torch.cuda.set_device(dev)
    ctx = wb.Context(local_rank)
    ctx.set_table_mode(args.table_mode)
    wl["table_mode"] = args.table_mode
    wl["exchange"] = args.exchange
    lo, hi = n_rows * rank // world, n_rows * (rank + 1) // world
    if wl["kind"] == "bins":
        wl["rows_total"] = n_rows
        job = BinsJob(ctx, wl, lo, hi, world, dist, dev, rank)
    elif wl["kind"] == "pushdown":
        if world > 1:
            raise SystemExit("the pushdown workload runs on one GPU (its per-rank groups are not merged)")
        wl["rows_total"] = n_rows
        job = PushdownJob(ctx, wl, lo, hi, world, dist, dev)
    else:
        job = (DenseJob if wl["kind"] == "dense" else HashJob)(ctx, wl, lo, hi, world, dist, dev)
    n_local = job.n_local
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()

    small = n_local * job.bpr <= 256 << 20
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if small else None

    def barrier():
        if dist is not None:
            dist.barrier()

    # the ranks enter every phase together: a step's exchange waits (bounded) for the other ranks
    barrier()
    for _ in range(args.warmup):
        if flush is not None:
            flush.zero_()
        job.step(job.inputs)
    ctx.sync()
    torch.cuda.synchronize()

    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        uuid = None
    clocks = ClockSampler(uuid)
    clocks.start()

    launches0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    ctx.profile(True)
    kbytes = 0
    ev0.record(stream)
    for _ in range(args.steps):
        if flush is not None:
            flush.zero_()
        job.step(job.inputs)
        kbytes += job.kernel_bytes()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ctx.profile(False)
    launches = ctx.launches - launches0
    kms, klaunches = ctx.kernel_time_ms()
    ctx.sync()  # surfaces deferred device errors (a key out of range, a full table)
    ms = ev0.elapsed_time(ev1)

    # ---- end to end through the public API, host buffers in pinned memory
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else max(3, min(args.steps, 10))
    extra = job.extra(args) if hasattr(job, "extra") else {}
    host_in = []
    for t in job.inputs:
        h = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        host_in.append(h)
    h2d_all = sum(h.numel() * h.element_size() for h in host_in)
    dev_in = [torch.empty_like(t) for t in job.inputs]
    job.inputs = None
    host_out = {}
    d2h = [0]
    h2d_step = [h2d_all]

    def e2e_step():
        if hasattr(job, "e2e_copy"):
            h2d_step[0] = job.e2e_copy(dev_in, host_in)
        else:
            for d, h in zip(dev_in, host_in):
                d.copy_(h, non_blocking=True)
        job.step(dev_in)
        d2h[0] = job.read_result(host_out)

    torch.cuda.synchronize()
    barrier()  # pinning the host copies takes each rank its own time
    e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = ev0.elapsed_time(ev1)
    ctx.sync()
    clk = clocks.stop()

    # ---- parity of the last step's result (outside every timed region)
    check = None
    if not args.no_check and hasattr(job, "check"):
        check = job.check(dev_in, dist, world)
        if dist is not None:
            okt = torch.tensor([1.0 if check.get("ok") else 0.0], device=dev)
            dist.all_reduce(okt, op=dist.ReduceOp.MIN)
            check["ok_all_ranks"] = bool(okt.item() == 1.0)

    # ---- max over ranks
    kern_gbs = kbytes / args.steps / (kms / max(klaunches, 1) / 1e3) / 1e9 if kms > 0 else 0.0
    t = torch.tensor([ms, e2e_ms, -kern_gbs, float(launches), float(h2d_step[0]), float(d2h[0])], dtype=torch.float64,
                     device=dev)
    if dist is not None:
        mx = t[:3].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t[3:].clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        t = torch.cat([mx, sm])
    ms_max, e2e_ms_max, neg_ach, launches_total, h2d_total, d2h_total = t.tolist()
    achieved = -neg_ach  # the slowest rank's kernel bandwidth
    if hasattr(getattr(job, "sharded", None), "finish"):
        torch.cuda.synchronize()
        job.sharded.finish()

    if rank != 0:
        return
    bpr = job.bpr
    value = n_rows * args.steps / (ms_max / 1e3)
    peak, peak_kind = measured_peak()
    tm, tsrc = traffic_model(args.workload)
    line = base_line(args, wl, n_rows, world)
    if getattr(job, "exchange", None):
        line["config"]["exchange"] = job.exchange
    line.update({
        "value": value,
        "ms_per_step": ms_max / args.steps,
        "impl": "ours",
        "e2e": {"value": n_rows * e2e_steps / (e2e_ms_max / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": int(h2d_total), "d2h_bytes_per_step": int(d2h_total), "steps": e2e_steps},
        "gpu_launches": int(launches_total),
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else
                           "fallback 6.65 TB/s",
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": (tm[0] * n_local + tm[1]) if tm else None,
            "traffic_source": tsrc,
            "kernel": job.kernel,
            "algorithmic_bytes_per_launch": kbytes / args.steps,
            "kernel_ms_avg": kms / max(klaunches, 1),
        },
        "hbm_gbs_job": n_rows * bpr / (ms_max / args.steps / 1e3) / 1e9,
        "clocks": clk,
        "device": ctx.name,
    })
    line.update(extra)
    if check is not None:
        line["check"] = check
    if world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        sample = cpu_sample_rows(wl, args.cpu_seconds, threads, n_rows)
        cols = host_inputs(wl, 0, sample)
        t0 = time.perf_counter()
        cpu_groupby(wl, cols, threads)
        dt = time.perf_counter() - t0
        how = ("exact Kulisch groupby" if wl["kind"] == "dense" else "sort-based exact groupby of int64 keys")
        line["cpu_baseline"] = {"value": sample / dt, "unit": "rows/s", "cores": threads, "kind": "port",
                                "sample": f"first {sample} rows of the workload, {how} "
                                          f"(oracle port of the reference's CPU path), {threads} threads",
                                "cpu_model": cpu_model(), "nproc": os.cpu_count()}
        if wl["kind"] != "bins":
            line["cpu_baseline"]["single_thread"] = single_thread_baseline(wl, n_rows)
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    wl = dict(WORKLOADS[args.workload])
    n_rows = args.rows or wl["rows"]
    if args.ids is not None and "ids" in wl:
        wl["ids"] = args.ids
        wl["desc"] += f" (distinct ids overridden: {args.ids})"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            print(json.dumps({"error": "launch with torch.distributed.run for --gpus > 1"}))
            sys.exit(2)
    dist = None
    if args.impl == "reference":
        run_reference(args, wl, n_rows, world, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist_mod

        torch.cuda.set_device(local_rank)
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device(f"cuda:{local_rank}"))
        dist = dist_mod
    try:
        run_ours(args, wl, n_rows, world, rank, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
