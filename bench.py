#!/usr/bin/env python
"""Groupby-aggregate throughput on B200: rows/s and HBM GB/s vs the measured peak.

Default workload (the low-cardinality sharded configuration): 1,000,000,000 rows,
int32 keys uniform in [0,256), f64 values ~U(-1,1); count/sum/min/max/mean/var per
key.  Rows are split evenly over N GPUs (one process per GPU, launched by
torch.distributed.run); each GPU reduces its shard to a mergeable per-group state
table, the tables are all-gathered over NCCL and folded in rank order.

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
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "groupby-agg rows/s and HBM GB/s (frac of ~8 TB/s) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    # name: rows, groups, value model, seed, description
    "lowcard": dict(rows=1_000_000_000, groups=256, values=("uniform", -1.0, 1.0), nonfinite=None, seed=0,
                    desc="low-cardinality sharded: 1,000,000,000 rows; int32 key uniform in [0,256); "
                         "f64 value ~U(-1,1); sum/count/min/max/mean/var; rows split evenly over the GPUs, "
                         "partial tables all-gathered over NCCL and merged"),
    "cpu-ref": dict(rows=1_000_000, groups=1000, values=("normal", 0.0, 1.0), nonfinite=None, seed=0,
                    desc="1,000,000 rows; int32 key uniform in [0,1000); f64 value ~N(0,1); "
                         "sum/count/min/max/mean/var; seed 0"),
    "stress-1k": dict(rows=200_000_000, groups=1000, values=("normal", 1e9, 1e-3), nonfinite=(0.01, 0.001), seed=0,
                      desc="200,000,000 rows; int32 key uniform in [0,1000); f64 value 1e9 + N(0,1e-3), 1% NaN, "
                           "0.1% +-inf; count/mean/var/min/max"),
}
BYTES_PER_ROW = 12  # 4 B key + 8 B value, each column read once


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


def traffic_per_row():
    """dram bytes per row of the main kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None, None
    try:
        d = json.loads(p.read_text())["dense_moments_kernel"]
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


def host_inputs(wl, start, count):
    """The workload's rows [start, start+count) generated on the host (same bits as the device generator
    for keys and uniform values)."""
    import oracle

    keys = oracle.gen_keys_uniform(count, wl["groups"], wl["seed"], start)
    kind, a, b = wl["values"]
    if kind == "uniform":
        vals = oracle.gen_values_uniform(count, a, b, wl["seed"], start)
    else:
        vals = oracle.gen_values_normal(count, a, b, wl["seed"], start)
    if wl["nonfinite"]:
        vals = oracle.inject_nonfinite(vals, wl["nonfinite"][0], wl["nonfinite"][1], wl["seed"], start)
    return keys, vals


def cpu_sample_rows(wl, target_s, threads):
    """Rows the oracle processes in about target_s seconds on `threads` threads (calibrated)."""
    import oracle

    n0 = min(2_000_000, wl["rows"])
    k, v = host_inputs(wl, 0, n0)
    t0 = time.perf_counter()
    oracle.moments_grouped_mt(v, k, wl["groups"], threads=threads)
    rate = n0 / (time.perf_counter() - t0)
    return min(max(n0, int(rate * target_s)), wl["rows"], 200_000_000)


def base_line(args, wl, n_rows, world):
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
        "config": {
            "workload": wl["desc"],
            "rows": n_rows,
            "n_groups": wl["groups"],
            "bytes_per_row": BYTES_PER_ROW,
            "parallelism": f"row-shards x{world}",
            "l2": "inputs (12 B/row) far larger than the 126 MB L2; no flush needed between steps"
            if n_rows * BYTES_PER_ROW > 1 << 30 else "inputs smaller than L2: L2 flushed between steps",
        },
    }


# ---------------------------------------------------------------------------------
# the reference arm: the reference's CPU groupby (oracle port) on the host cores
# ---------------------------------------------------------------------------------

def run_reference(args, wl, n_rows, world, rank):
    if rank != 0:
        return
    import oracle

    threads = cpu_threads()
    per_step_s = max(2.0, min(20.0, 150.0 / max(1, args.steps + args.warmup)))
    sample = cpu_sample_rows(wl, per_step_s, threads)
    k, v = host_inputs(wl, 0, sample)
    for _ in range(args.warmup):
        oracle.moments_grouped_mt(v, k, wl["groups"], threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.moments_grouped_mt(v, k, wl["groups"], threads=threads)
    dt = time.perf_counter() - t0
    value = sample * args.steps / dt
    line = base_line(args, wl, n_rows, world)
    line.update({
        "impl": "reference",
        "value": value,
        "ms_per_step": dt * 1000.0 / args.steps,
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"first {sample} rows of the workload per step (exact Kulisch groupby, "
                                   f"per-thread registers merged in row-range order)"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------

def run_ours(args, wl, n_rows, world, rank, local_rank, dist):
    import torch

    import winrapids_b200 as wb

    dev = torch.device(f"cuda:{local_rank}")
    torch.cuda.set_device(dev)
    ctx = wb.Context(local_rank)
    G = wl["groups"]
    lo, hi = n_rows * rank // world, n_rows * (rank + 1) // world
    n_local = hi - lo
    stream = torch.cuda.current_stream()

    # inputs resident in HBM, generated where they live
    dk = torch.empty(n_local, dtype=torch.int32, device=dev)
    dv = torch.empty(n_local, dtype=torch.float64, device=dev)
    ctx.gen_keys_uniform(dk, G, wl["seed"], lo)
    kind, a, b = wl["values"]
    if kind == "uniform":
        ctx.gen_values_uniform(dv, a, b, wl["seed"], lo)
    else:
        ctx.gen_values_normal(dv, a, b, wl["seed"], lo)
    if wl["nonfinite"]:
        ctx.gen_inject_nonfinite(dv, wl["nonfinite"][0], wl["nonfinite"][1], wl["seed"], lo)
    out = ctx.alloc_moments(G)
    st_local = torch.empty(ctx.state_bytes(G) // 8, dtype=torch.float64, device=dev)
    gathered = torch.empty(world * st_local.numel(), dtype=torch.float64, device=dev)
    torch.cuda.synchronize()

    small = n_local * BYTES_PER_ROW <= 256 << 20
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if small else None

    def step(keys, vals):
        if world == 1:
            ctx.groupby_dense(keys, vals, G, out=out, sync=False)
        else:
            ctx.groupby_dense_state(keys, vals, G, row_offset=lo, state=st_local)
            dist.all_gather_into_tensor(gathered, st_local)
            ctx.merge_states(gathered, world, G, out=out)

    def barrier():
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        if flush is not None:
            flush.zero_()
        step(dk, dv)
    ctx.sync()
    torch.cuda.synchronize()

    uuid = None
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
    ev0.record(stream)
    for _ in range(args.steps):
        if flush is not None:
            flush.zero_()
        step(dk, dv)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ctx.profile(False)
    launches = ctx.launches - launches0
    kms, klaunches = ctx.kernel_time_ms()
    ctx.sync()  # surfaces deferred device errors (e.g. a key out of range)
    ms = ev0.elapsed_time(ev1)

    # ---- end to end through the public API, host buffers in pinned memory
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else max(3, min(args.steps, 10))
    hk = torch.empty(n_local, dtype=torch.int32, pin_memory=True)
    hv = torch.empty(n_local, dtype=torch.float64, pin_memory=True)
    hk.copy_(dk)
    hv.copy_(dv)
    hout = {f: torch.empty(G, dtype=torch.float64, pin_memory=True) for f in out}
    ek = torch.empty_like(dk)
    ev = torch.empty_like(dv)
    del dk, dv

    def e2e_step():
        ek.copy_(hk, non_blocking=True)
        ev.copy_(hv, non_blocking=True)
        step(ek, ev)
        for f in out:
            hout[f].copy_(out[f], non_blocking=True)

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

    # ---- max over ranks
    t = torch.tensor([ms, e2e_ms, -(n_local * BYTES_PER_ROW / (kms / max(klaunches, 1) / 1e3) / 1e9 if kms > 0 else 0.0),
                      float(launches)], dtype=torch.float64, device=dev)
    if dist is not None:
        mx = t[:3].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t[3:].clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        t = torch.cat([mx, sm])
    ms_max, e2e_ms_max, neg_ach, launches_total = t.tolist()
    achieved = -neg_ach  # the slowest rank's kernel bandwidth

    if rank != 0:
        return
    value = n_rows * args.steps / (ms_max / 1e3)
    peak, peak_kind = measured_peak()
    tpr, tsrc = traffic_per_row()
    line = base_line(args, wl, n_rows, world)
    line.update({
        "value": value,
        "ms_per_step": ms_max / args.steps,
        "impl": "ours",
        "e2e": {"value": n_rows * e2e_steps / (e2e_ms_max / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": n_rows * BYTES_PER_ROW,
                "d2h_bytes_per_step": world * len(out) * G * 8, "steps": e2e_steps},
        "gpu_launches": int(launches_total),
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else
                           "fallback 6.65 TB/s",
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": (tpr[0] * n_local + tpr[1]) if tpr else None,
            "traffic_source": tsrc,
            "kernel": "dense_moments_kernel",
            "algorithmic_bytes_per_launch": n_local * BYTES_PER_ROW,
            "kernel_ms_avg": kms / max(klaunches, 1),
        },
        "hbm_gbs_job": n_rows * BYTES_PER_ROW / (ms_max / args.steps / 1e3) / 1e9,
        "clocks": clk,
        "device": ctx.name,
    })
    if world == 1 and not args.no_cpu_baseline:
        import oracle

        threads = cpu_threads()
        sample = cpu_sample_rows(wl, args.cpu_seconds, threads)
        k, v = host_inputs(wl, 0, sample)
        t0 = time.perf_counter()
        oracle.moments_grouped_mt(v, k, G, threads=threads)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": sample / dt, "unit": "rows/s", "cores": threads, "kind": "port",
                                "sample": f"first {sample} rows of the workload, exact Kulisch groupby "
                                          f"(oracle port of the reference's CPU path), {threads} threads"}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    wl = dict(WORKLOADS[args.workload])
    n_rows = args.rows or wl["rows"]
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
