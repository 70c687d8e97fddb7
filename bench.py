#!/usr/bin/env python
"""forge-sort B200 benchmark (driver contract: one JSON line on rank 0).

Workload: sort 2^32 u32 keys -- elements [0, 2^32) of
the seed-42 xorshift64 stream, uniform over [0, 2^32) -- partitioned over N
GPUs (strong scaling: total keys fixed).  N = 1 is the single-GPU LSD radix
sort; N > 1 is the sample sort (regular-sampling splitters, one fused
partition + exchange pass into the peers' inboxes over NVLink, local radix
sort).

  value : sorted Mkeys/s, inputs resident in HBM, out-of-place device sort
          (the pristine input is re-read every step; 16 GiB >> 126 MB L2)
  e2e   : the same through the host API: pinned host keys -> device -> sort
          -> pinned host output, every step (streaming calls; the synchronous
          call is reported beside it)
  roofline : dominant kernel = the stable-rank scatter pass, algorithmic
          bytes per key = 2 x key bytes (read + write), timed live with CUDA
          events on the library's stream
  cpu_baseline : the oracle's parallel sort (C++ stand-in for rayon
          par_sort_unstable) on a bounded sample, rank 0 at N = 1

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --suite     # every BASELINE config on one GPU, one JSON
                              # line each (not part of the driver contract)
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gpu-forge_b200"))
sys.path.insert(0, ROOT)

METRIC = "sorted Mkeys/s (u32, 2^32 keys, sample sort over N B200)"
UNIT = "Mkeys/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--log2n", type=int, default=32, help="total keys = 2^log2n")
    p.add_argument("--dist", choices=["uniform", "skew"], default="uniform")
    p.add_argument("--dtype", choices=["u32", "u64"], default="u32")
    p.add_argument("--op", choices=["keys", "argsort", "pairs"], default="keys",
                   help="N > 1: keys-only sample sort (the headline), or the payload forms")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--profile-steps", type=int, default=3)
    p.add_argument("--suite", action="store_true", help="time every BASELINE config on one GPU")
    p.add_argument("--only", default="", help="--suite: run only the rows whose config or op contains this")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def config(args, world):
    what = {"keys": "sort", "argsort": "argsort (u32 global positions) of", "pairs": "sort_pairs (u32 values) of"}
    return {
        "workload": f"configs[4]: {what[getattr(args, 'op', 'keys')]} {args.dtype} keys, "
                    f"{'uniform' if args.dist == 'uniform' else '70% in one 2^20 range'}"
                    f", total 2^{args.log2n} keys partitioned over N GPUs",
        "keys_total": 1 << args.log2n,
        "keys_per_gpu": (1 << args.log2n) // world,
        "key_type": args.dtype,
        "generator": "xorshift64 seed 42 (element i = state after i+1 steps; shard r = elements [r*m,(r+1)*m))",
        "parallelism": f"sample sort x{world}" if world > 1 else "single GPU LSD radix sort",
        "l2": "inputs (>= 2 GiB per GPU) larger than the 126 MB L2; no flush needed",
    }


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampled every 50 ms while the timed region runs (the
    sampler is running before the region starts)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
            t_end = time.time() + 5.0  # wait for the first sample
            while time.time() < t_end and self.proc.poll() is None and os.fstat(self.f.fileno()).st_size == 0:
                time.sleep(0.01)
            self.f.seek(0, os.SEEK_END)
            self.skip = self.f.tell()  # samples taken before the region are not counted
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.proc or not self.f:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.f.seek(getattr(self, "skip", 0))
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "samples": len(sm), "reasons": sorted(reasons)}


def measured_peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(dtype: str, kernel: str = "k_scatter, stable"):
    """Per-key DRAM bytes (read + write) of one launch of `kernel` from the
    committed ncu summaries (profiles/*_traffic.json: the stable k_scatter,
    the histogram fill), scaled by the caller; None if absent."""
    name = "k_hf_local_traffic.json" if kernel.startswith("k_hf_local") else "k_scatter_stable_traffic.json"
    if not kernel.startswith(("k_hf_local", "k_scatter, stable")):
        return None, None
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            d = json.load(f)
        return d[dtype]["dram_bytes_per_key"], d[dtype]
    except Exception:
        return None, None


# ------------------------------------------------------------------ CPU leg
def cpu_sample_time(dtype: str, sample_n: int, threads: int, reps: int):
    """Seconds per sort of `sample_n` keys by the oracle's CPU sort."""
    from oracle import oracle as orc
    x = orc.gen("u32" if dtype == "u32" else "u64", sample_n, seed=42)
    best = []
    for _ in range(reps):
        t0 = time.perf_counter()
        if threads == 1:
            orc.sort_keys(x, dtype)
        else:
            orc.par_sort_keys(x, dtype, threads)
        best.append(time.perf_counter() - t0)
    best.sort()
    return best[len(best) // 2]


def cpu_baseline(dtype: str):
    from oracle import oracle as orc
    threads = orc.max_threads()
    n_par = 1 << 26
    t_par = cpu_sample_time(dtype, n_par, threads, 3)
    n_one = 1 << 24
    t_one = cpu_sample_time(dtype, n_one, 1, 1)
    return {
        "value": round(n_par / t_par / 1e6, 2), "unit": UNIT, "cores": threads, "kind": "port",
        "sample": f"2^26 {dtype} keys (same generator), median of 3; __gnu_parallel::sort on ordered bits "
                  "(C++ stand-in for rayon par_sort_unstable)",
        "single_thread": {"value": round(n_one / t_one / 1e6, 2), "unit": UNIT, "cores": 1,
                          "sample": f"2^24 {dtype} keys, std::sort (stand-in for sort_unstable)"},
    }


def run_reference(args):
    """--impl reference: the reference's CPU path (oracle port) on host cores."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle as orc
    threads = orc.max_threads()
    sample_n = 1 << 26
    dt = args.dtype
    x = orc.gen("u32" if dt == "u32" else "u64", sample_n, seed=42)
    for _ in range(args.warmup):
        orc.par_sort_keys(x, dt, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.par_sort_keys(x, dt, threads)
    dt_s = (time.perf_counter() - t0) / max(args.steps, 1)
    v = round(sample_n / dt_s / 1e6, 2)
    line = {
        "metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt_s * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dt,
        "data": "synthetic",
        # same workload and metric as our arm; each step sorts a bounded
        # 2^26-key sample of it (the full 2^32 keys would take minutes a step)
        "config": {**config(args, world), "keys_per_step": sample_n,
                   "parallelism": f"CPU, {threads} host threads (__gnu_parallel::sort)",
                   "sample": f"first 2^26 keys of the 2^{args.log2n}-key input, sorted each step"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"each step sorts 2^26 keys of the same stream with __gnu_parallel::sort "
                                   "(C++ restatement of the reference's CPU path; Rust toolchain absent)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ ours
# Kernels of one sort as the library times them (fs_last_kernel_times), with
# the algorithmic bytes each moves per key.  Two layouts:
#   LSD chain (2 + 2P + 1 entries): first count, plan, (count + scan,
#     scatter) per pass, finalize
#   keys-only 32-bit sorts from FORGESORT_H16_MIN_KEYS keys (10 entries):
#     first count (digit 2), plan, scan + scatter (digit 2, unstable),
#     count + scan + scatter (digit 3, stable), group bounds, group fill,
#     large groups, finalize
def kernel_table(times, kb):
    P = kb
    if len(times) == 10 and kb == 4:
        return [
            ("k_first_count (digit-2 slice counts + OR/AND of all keys, reads every key)", times[0], kb),
            ("k_scatter, unstable ranking (digit 2, first pass of the top 16 bits)", times[3], 2 * kb),
            ("k_count + k_slice_scan (digit 3)", times[4], kb),
            ("k_scatter, digit 3 (keeps digit-2 order: atomic ranks where a warp round agrees on digit 2)",
             times[5], 2 * kb),
            ("k_hf_local (histogram fill: each top-16-bit group sorted by counting its low 16 bits; "
             "reads and writes every key)", times[7], 2 * kb),
            ("k_hf_bounds + k_hf_plan (group starts)", times[6], 0),
            ("k_hf_big_* (groups over 126975 keys)", times[8], 0),
        ]
    rows = [("k_first_count (digit-0 slice counts + OR/AND of all keys, reads every key)", times[0], kb)]
    rows.append(("k_scatter, unstable ranking (first executed pass, keys only)", times[3], 2 * kb))
    for p in range(1, P):
        rows.append(("k_count + k_slice_scan (per-slice digit counts, reads every key)", times[2 + 2 * p], kb))
        rows.append(("k_scatter, stable ranking (one 8-bit LSD pass: rank, stage, scatter)", times[3 + 2 * p],
                     2 * kb))
    return rows


def kernel_roofline(sorter, step, stream, m, kb, ms, profile_steps, dt):
    """Roofline of the dominant kernel (most device time per sort among the
    kernels that move keys), every kernel's share, and the whole sort against
    the K(1 + 2P) bytes-per-key model."""
    import torch

    sorter.set_kernel_timing(True)
    runs = []
    with torch.cuda.stream(stream):
        for _ in range(max(profile_steps, 1)):
            step()
            runs.append(sorter.last_kernel_times())
    sorter.set_kernel_timing(False)
    avg = [sum(r[i] for r in runs) / len(runs) for i in range(len(runs[0]))]
    peak, peak_kind = measured_peak_hbm()
    frac = lambda b, t_ms: round(b / (t_ms * 1e-3) / 1e9 / peak, 4) if t_ms > 0 else None
    rows = kernel_table(avg, kb)
    # merge repeated kernels (the LSD chain's passes) by name
    merged = {}
    for name, t, bpk in rows:
        e = merged.setdefault(name, {"ms": 0.0, "launches": 0, "bpk": bpk})
        e["ms"] += t
        e["launches"] += 1
    dom_name = max((k for k in merged if merged[k]["bpk"] > 0), key=lambda k: merged[k]["ms"])
    dom = merged[dom_name]
    launch_ms = dom["ms"] / dom["launches"]
    alg = m * dom["bpk"]
    achieved = alg / (launch_ms * 1e-3) / 1e9
    tr_per_key, tr_rec = committed_traffic(dt, dom_name)
    P = kb
    total = sum(e["ms"] for e in merged.values())
    roofline = {
        "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
        "traffic": round(tr_per_key * m) if tr_per_key else None,
        "kernel": dom_name,
        "alg_bytes_per_launch": alg,
        "launch_ms": round(launch_ms, 4),
        "kernels": [{"kernel": k, "launches": e["launches"], "ms": round(e["ms"], 4),
                     "share": round(e["ms"] / total, 4) if total else None,
                     "frac": frac(m * e["bpk"] * e["launches"], e["ms"]) if e["bpk"] else None}
                    for k, e in merged.items()],
        "sort_alg_bytes_per_key": kb * (1 + 2 * P),
        "sort_frac": frac(m * kb * (1 + 2 * P), ms),
        "sort_bytes_moved_per_key": sum(e["bpk"] * e["launches"] for e in merged.values()),
    }
    if tr_rec:
        roofline["traffic_source"] = tr_rec.get("source")
    return roofline


def run_ours(args):
    import torch
    import torch.distributed as tdist

    import forge_sort
    from forge_sort import _lib

    rank, world, local = dist_env()
    if world > 1:
        return run_multi(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(device=dev)
    sorter = forge_sort.GpuSorter.with_context(local, stream)
    L = _lib.load()
    dt = args.dtype
    kb = 4 if dt == "u32" else 8
    n_total = 1 << args.log2n
    m = n_total // world
    tdt = torch.int32 if kb == 4 else torch.int64
    keys_in = torch.empty(m, dtype=tdt, device=dev)
    keys_out = torch.empty(m, dtype=tdt, device=dev)
    gen = {"u32": _lib.GEN_U32, "u64": _lib.GEN_U64}[dt]
    if args.dist == "skew":
        gen = _lib.GEN_SKEW_U32
    rc = L.fs_generate(gen, 42, rank * m, m, keys_in.data_ptr(), stream.cuda_stream)
    assert rc == 0, rc
    stream.synchronize()

    def step():
        sorter.sort_device_copy(dt, keys_in.data_ptr(), keys_out.data_ptr(), m, sync=False)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        sorter.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk:
            torch.cuda.synchronize()
            t0.record(stream)
            for _ in range(args.steps):
                step()
            t1.record(stream)
            t1.synchronize()
            sorter.synchronize()  # surfaces any device-side failure
        ms = t0.elapsed_time(t1) / args.steps
    clocks = clk.summary()
    launches_per_step = sorter.last_launch_count()

    # correctness spot check of the timed output (sortedness + checksum-free)
    tail = keys_out[: 1 << 20].cpu().numpy().view("u4" if kb == 4 else "u8")
    assert (tail[1:] >= tail[:-1]).all(), "bench output not sorted"

    roofline = kernel_roofline(sorter, step, stream, m, kb, ms, args.profile_steps, dt)

    value = m * world / (ms * 1e-3) / 1e6

    e2e = None
    if not args.no_e2e:
        h_in = torch.empty(m, dtype=tdt, pin_memory=True)
        h_out = torch.empty(m, dtype=tdt, pin_memory=True)
        h_in.copy_(keys_in.cpu())
        del keys_out
        torch.cuda.empty_cache()
        ew = min(args.warmup, 3)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # streaming API: each step copies its keys in, sorts and copies the
        # result out; consecutive steps overlap their copies
        for _ in range(ew):
            sorter.host_sort_copy_async_ptr(dt, h_in.data_ptr(), h_out.data_ptr(), m)
        sorter.synchronize()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            sorter.host_sort_copy_async_ptr(dt, h_in.data_ptr(), h_out.data_ptr(), m)
        sorter.synchronize()  # the stream now waits for every step's copy back
        e1.record(stream)
        e1.synchronize()
        ems = e0.elapsed_time(e1) / args.steps
        chk = h_out[: 1 << 20].numpy().view("u4" if kb == 4 else "u8")
        assert (chk[1:] >= chk[:-1]).all()
        # one synchronous call at a time (fs_host_sort_keys_copy), for reference
        h_out.zero_()
        sorter.host_sort_copy_ptr(dt, h_in.data_ptr(), h_out.data_ptr(), m)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            sorter.host_sort_copy_ptr(dt, h_in.data_ptr(), h_out.data_ptr(), m)
        e1.record(stream)
        e1.synchronize()
        sms = e0.elapsed_time(e1) / args.steps
        chk = h_out[: 1 << 20].numpy().view("u4" if kb == 4 else "u8")
        assert (chk[1:] >= chk[:-1]).all()
        e2e = {"value": round(m * world / (ems * 1e-3) / 1e6, 2), "unit": UNIT,
               "h2d_bytes_per_step": m * kb, "d2h_bytes_per_step": m * kb,
               "ms_per_step": round(ems, 3),
               "api": "fs_host_sort_keys_copy_async, one call per step (pinned host in/out; a step's copy in "
                      "overlaps the previous step's sort and copy out)",
               "single_call": {"value": round(m * world / (sms * 1e-3) / 1e6, 2), "ms_per_step": round(sms, 3),
                               "api": "fs_host_sort_keys_copy (synchronous)"}}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(dt)

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dt, "data": "synthetic", "config": config(args, world),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
        "gpu_launches": launches_per_step * args.steps,
        "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    sorter.close()


def run_multi(args):
    """N > 1: the sample sort, one process per GPU (torchrun), NCCL all-to-all."""
    import datetime

    import torch
    import torch.distributed as tdist

    import forge_sort
    from forge_sort import _lib
    from forge_sort.samplesort import CudaOps, SampleSorter

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    stream = torch.cuda.Stream(device=dev)
    sorter = forge_sort.GpuSorter.with_context(local, stream)
    L = _lib.load()
    dt = args.dtype
    kb = 4 if dt == "u32" else 8
    n_total = 1 << args.log2n
    m = n_total // world
    tdt = torch.int32 if kb == 4 else torch.int64
    keys_in = torch.empty(m, dtype=tdt, device=dev)
    gen = {"u32": _lib.GEN_U32, "u64": _lib.GEN_U64}[dt]
    if args.dist == "skew":
        gen = _lib.GEN_SKEW_U32
    assert L.fs_generate(gen, 42, rank * m, m, keys_in.data_ptr(), stream.cuda_stream) == 0
    op = args.op
    vals_in = None
    if op == "pairs":  # values: a scrambled global position per key
        vals_in = ((torch.arange(m, dtype=torch.int64, device=dev) + rank * m) * 2654435761 & 0xFFFFFFFF).to(torch.int32)
    stream.synchronize()
    ss = SampleSorter(CudaOps(sorter, torch), dtype=dt)
    vb = 0 if op == "keys" else 4  # payload bytes per key

    def step():
        # sync=False: a step's local sort stays in flight; the next step's one
        # host wait (for the all-gathered bucket counts) follows it on the
        # stream, and ss.synchronize() after the timed loop reports errors
        if op == "keys":
            return ss.sort(keys_in, gpos_base=rank * m, sync=False)
        if op == "argsort":
            return ss.sort_with_positions(keys_in, gpos_base=rank * m, sync=False)
        return ss.sort_pairs(keys_in, vals_in, gpos_base=rank * m, sync=False)

    def timed(fn, steps):
        tdist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        out = None
        for _ in range(steps):
            out = fn()
        e1.record(stream)
        e1.synchronize()
        ss.synchronize()  # device-side errors of the last step
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)  # the job is as slow as its slowest rank
        tdist.barrier()
        return float(t.item()), out

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            out = step()
        del out
        with Clocks(local) as clk:
            ms, out = timed(step, args.steps)
    clocks = clk.summary()

    # correctness of the timed output: sorted pieces, ordered across ranks,
    # all keys accounted for; with a payload, the values of this rank's own
    # keys match the input
    if op != "keys":
        out, vout = out
        if op == "argsort":
            pos = vout.to(torch.int64) & 0xFFFFFFFF
            own = (pos >= rank * m) & (pos < (rank + 1) * m)
            assert bool((keys_in[pos[own] - rank * m] == out[own]).all()), "positions do not match the keys"
        del vout
    o = out.cpu().numpy().view("u4" if kb == 4 else "u8")
    assert (o[1:] >= o[:-1]).all(), "rank output not sorted"
    edge = torch.tensor([int(o[0]) if o.size else -1, int(o[-1]) if o.size else -1, o.size],
                        dtype=torch.float64, device=dev)
    edges = [torch.empty_like(edge) for _ in range(world)]
    tdist.all_gather(edges, edge)
    ev = [e.cpu().tolist() for e in edges]
    assert sum(int(e[2]) for e in ev) == n_total, "keys lost in the exchange"
    nonempty = [e for e in ev if e[2] > 0]
    assert all(a[1] <= b[0] for a, b in zip(nonempty, nonempty[1:])), "ranks out of order"
    recv = ss.last.recv_counts
    max_piece = max(int(e[2]) for e in ev)

    # dominant kernel: k_scatter of the local sort (the last call of a step)
    sorter.set_kernel_timing(True)
    with torch.cuda.stream(stream):
        step()
    t = sorter.last_kernel_times()
    sorter.set_kernel_timing(False)
    P = kb
    if op == "keys" and len(t) == 10 and kb == 4:  # histogram-fill form: the stable digit-3 pass
        pass_ms = [t[5]]
    else:
        pass_ms = [t[3 + 2 * p] for p in range(1, P)]  # stable passes (pass 0 of keys-only ranks unstably)
    pass_avg = sum(pass_ms) / len(pass_ms)
    peak, peak_kind = measured_peak_hbm()
    piece = out.numel()
    achieved = piece * 2 * (kb + vb) / (pass_avg * 1e-3) / 1e9
    # phase-summed roofline of the whole job (slowest rank holds max_piece):
    # bucket count + dispatch pass (3K; the dispatch's stores are the
    # exchange), local sort (K(1+2P) + K(P-1) counts) over HBM, and (G-1)/G
    # of the keys over NVLink at the measured 770 GB/s per direction
    nvlink = 770.0
    vread = 4 if op == "pairs" else 0  # argsort's positions are made in the dispatch
    hbm_b = m * (3 * kb + vread + vb) + max_piece * (kb * (1 + 2 * P) + kb * (P - 1) + vb * 2 * P)
    t_roof = hbm_b / (peak * 1e9) + m * (kb + vb) * (world - 1) / world / (nvlink * 1e9)
    roofline = {
        "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
        "kernel": "k_scatter, stable ranking (local sort pass)", "alg_bytes_per_launch": piece * 2 * (kb + vb),
        "pass_ms": round(pass_avg, 4),
        "job_roofline_ms": round(t_roof * 1e3, 3), "job_frac": round(t_roof * 1e3 / ms, 4),
        "job_model": "HBM: bucket count K + dispatch pass 2K (its stores land in the peers' inboxes) + local sort K(1+2P)+K(P-1) per key, plus V per key for each payload read and write; NVLink (G-1)/G*(K+V) at 770 GB/s",
    }
    value = n_total / (ms * 1e-3) / 1e6

    e2e = None
    if not args.no_e2e:
        h_in = torch.empty(m, dtype=tdt, pin_memory=True)
        h_in.copy_(keys_in.cpu())
        h_out = torch.empty(max_piece + (1 << 20), dtype=tdt, pin_memory=True)
        if op != "keys":
            hv_out = torch.empty(max_piece + (1 << 20), dtype=torch.int32, pin_memory=True)
        if op == "pairs":
            hv_in = torch.empty(m, dtype=torch.int32, pin_memory=True)
            hv_in.copy_(vals_in.cpu())

        def e2e_step():
            d_in = torch.empty(m, dtype=tdt, device=dev)
            d_in.copy_(h_in, non_blocking=True)
            if op == "keys":
                r = ss.sort(d_in, gpos_base=rank * m)
                h_out[: r.numel()].copy_(r, non_blocking=True)
                return r.numel()
            if op == "argsort":
                v = ss.argsort(d_in, gpos_base=rank * m)
            else:
                dv = torch.empty(m, dtype=torch.int32, device=dev)
                dv.copy_(hv_in, non_blocking=True)
                r, v = ss.sort_pairs(d_in, dv, gpos_base=rank * m)
                h_out[: r.numel()].copy_(r, non_blocking=True)
            hv_out[: v.numel()].copy_(v, non_blocking=True)
            return v.numel()

        with torch.cuda.stream(stream):
            for _ in range(min(args.warmup, 3)):
                e2e_step()
            ems, got = timed(e2e_step, args.steps)
        h2d = m * kb + (m * 4 if op == "pairs" else 0)
        d2h = int(got) * ({"keys": kb, "argsort": 4, "pairs": kb + 4}[op])
        api = {"keys": "SampleSorter.sort", "argsort": "SampleSorter.argsort", "pairs": "SampleSorter.sort_pairs"}[op]
        e2e = {"value": round(n_total / (ems * 1e-3) / 1e6, 2), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(ems, 3), "api": f"{api} on pinned host shards (H2D, sort, D2H per rank)"}

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dt, "data": "synthetic", "config": config(args, world),
        "roofline": roofline, "cpu_baseline": None, "e2e": e2e, "clocks": clocks,
        "gpu_launches": (5 + 2 + 3 * P) * args.steps,  # count + dispatch chain, local sort 2 + 3P
        "balance": {"max_piece": max_piece, "mean_piece": n_total // world, "recv_counts_rank0": recv if rank == 0 else None},
        "op": op,
        "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    ss.close()
    sorter.close()
    tdist.barrier()
    tdist.destroy_process_group()


# ------------------------------------------------------------------ suite
SUITE = [  # (config, op, dtype, generator, n)
    ("configs[0]", "keys", "u32", "u32", 1 << 20),
    ("configs[1]", "keys", "u32", "u32", 1 << 24),
    ("configs[1]", "keys", "i32", "i32", 1 << 24),
    ("configs[1]", "keys", "f32", "f32_mix", 1 << 24),
    ("configs[2]", "keys", "u64", "u64", 1 << 26),
    ("configs[2]", "keys", "i64", "i64", 1 << 26),
    ("configs[2]", "keys", "f64", "f64_logu", 1 << 26),
    ("configs[2]", "argsort", "f32", "f32_mix", 1 << 24),
    ("configs[3]", "pairs", "u32", "zipf_u32", 1 << 28),
    ("1G u32", "keys", "u32", "u32", 1 << 30),
    ("configs[4] skewed", "keys", "u32", "skew_u32", 1 << 32),
    ("configs[4] u64", "keys", "u64", "u64", 1 << 30),
    ("configs[4] sample-sort kernels, 2 buckets", "dispatch", "u32", "u32", 1 << 28),
    ("configs[4] sample-sort kernels, 8 buckets", "dispatch", "u32", "u32", 1 << 28),
    ("small-n single CTA (gpu-search argsort_u64 path)", "keys", "u64", "u64", 4096),
    ("permutation apply (GpuGather) u32", "gather", "u32", "u32", 1 << 24),
]


def alg_bytes_per_key(op: str, kb: int, passes: int) -> int:
    """Bytes an LSD sort must move per key with `passes` executed digit
    passes: one read to count, then per pass the key read and written
    (argsort: plus the index, synthesised on the first pass; pairs: plus the
    u32 value read and written)."""
    if op == "keys":
        return kb * (1 + 2 * passes)
    if op == "argsort":
        return kb * (1 + 2 * passes) + 8 * passes - 4
    return kb * (1 + 2 * passes) + 8 * passes


def executed_passes(host, dt: str) -> int:
    """Digit passes that run: bytes of the order-transformed keys that vary."""
    import numpy as np
    from forge_sort.samplesort import ordered_bits
    o = ordered_bits(host, dt)
    varying = int(np.bitwise_or.reduce(o)) & ~int(np.bitwise_and.reduce(o))
    kb = 8 if dt in ("u64", "i64", "f64") else 4
    return sum(1 for b in range(kb) if (varying >> (8 * b)) & 0xff)


def run_suite(args):
    """Every BASELINE config on one GPU: device-resident sorts (CUDA events,
    median of the timed reps), plus the host-slice call (H2D + sort + D2H)
    and the zero-copy SortBuffer path where the reference reports them."""
    import numpy as np
    import torch

    import forge_sort
    from forge_sort import _lib
    from oracle import oracle as orc

    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(device=dev)
    sorter = forge_sort.GpuSorter.with_context(0, stream)
    L = _lib.load()
    peak, peak_kind = measured_peak_hbm()
    gen_dev = {"u32": _lib.GEN_U32, "u64": _lib.GEN_U64, "skew_u32": _lib.GEN_SKEW_U32}

    def timed(fn, reps):
        ts = []
        with torch.cuda.stream(stream):
            for _ in range(2):
                fn()
            sorter.synchronize()
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                e1.synchronize()
                ts.append(e0.elapsed_time(e1))
        sorter.synchronize()
        ts.sort()
        return ts[len(ts) // 2]

    for cfg, op, dt, gen, n in SUITE:
        if args.only and args.only not in cfg and args.only != op:
            continue
        kb = 8 if dt in ("u64", "i64", "f64") else 4
        tdt = torch.int32 if kb == 4 else torch.int64
        if gen in gen_dev:
            kin = torch.empty(n, dtype=tdt, device=dev)
            assert L.fs_generate(gen_dev[gen], 42, 0, n, kin.data_ptr(), stream.cuda_stream) == 0
            stream.synchronize()
            host = None
        else:
            host = orc.gen(gen, n, seed=42)
            kin = torch.from_numpy(np.ascontiguousarray(host).view(np.int32 if kb == 4 else np.int64)).to(dev)
        reps = max(3, min(20, (1 << 28) // n * 3))
        passes = executed_passes(host, dt) if host is not None else kb  # uniform device data: all vary
        bpk = alg_bytes_per_key(op, kb, passes) if op != "dispatch" else 3 * kb
        row = {"config": cfg, "op": op, "dtype": dt, "dist": gen, "n": n, "executed_passes": passes}
        if op == "keys":
            kout = torch.empty_like(kin)
            ms = timed(lambda: sorter.sort_device_copy(dt, kin.data_ptr(), kout.data_ptr(), n, sync=False), reps)
        elif op == "dispatch":
            # the sample sort's count + dispatch kernels on one GPU: splitters
            # at the bucket quantiles, every destination on this GPU (the
            # kernels are the same; over NVLink the stores go to peers)
            G = 2 if "2 buckets" in cfg else 8
            spl = np.array([(j << 32) // G for j in range(1, G)], dtype=np.uint64).astype(np.uint32)
            sk = torch.from_numpy(spl.view(np.int32)).to(dev)
            sg = torch.zeros(G - 1, dtype=torch.int64, device=dev)
            out = torch.empty_like(kin)
            cnt = sorter.partition_count(dt, kin.data_ptr(), n, 0, sk.data_ptr(), sg.data_ptr(), G - 1)
            dst = [out.data_ptr() + kb * sum(cnt[:b]) for b in range(G)]
            sorter.set_kernel_timing(True)
            kc, kd = [], []
            for _ in range(reps):
                sorter.partition_count(dt, kin.data_ptr(), n, 0, sk.data_ptr(), sg.data_ptr(), G - 1)
                kc.append(sorter.last_kernel_times()[0])
                sorter.partition_dispatch(dt, kin.data_ptr(), n, 0, sk.data_ptr(), sg.data_ptr(), G - 1, dst,
                                          sync=True)
                kd.append(sum(sorter.last_kernel_times()))
            sorter.set_kernel_timing(False)
            kc.sort()
            kd.sort()
            ms = kc[len(kc) // 2] + kd[len(kd) // 2]
            row["count_ms"] = round(kc[len(kc) // 2], 4)
            row["dispatch_ms"] = round(kd[len(kd) // 2], 4)
            row["count_frac"] = round(n * kb / (row["count_ms"] * 1e-3) / 1e9 / peak, 4)
            row["dispatch_frac"] = round(n * 2 * kb / (row["dispatch_ms"] * 1e-3) / 1e9 / peak, 4)
            head = out[: min(cnt[0], 1 << 20)].cpu().numpy().view(np.uint32)
            tail = out[n - min(cnt[-1], 1 << 20):].cpu().numpy().view(np.uint32)
            assert (head < spl[0]).all() and (tail >= spl[-1]).all(), "dispatch put keys in the wrong bucket"
        elif op == "gather":  # dst[i] = src[perm[i]]: random 4-byte reads, coalesced writes
            perm = torch.randperm(n, device=dev, dtype=torch.int64).to(torch.int32)
            dst = torch.empty_like(kin)
            ms = timed(lambda: sorter.gather_device(4, kin.data_ptr(), n, perm.data_ptr(), dst.data_ptr(), n,
                                                    sync=False), reps)
            bpk = 12  # index read + source read + destination write
            assert torch.equal(dst[:1000], kin[perm[:1000].to(torch.int64)])
        elif op == "argsort":
            idx = torch.empty(n, dtype=torch.int32, device=dev)
            ms = timed(lambda: sorter.argsort_device(dt, kin.data_ptr(), idx.data_ptr(), n, sync=False), reps)
        else:  # pairs through the zero-copy SortBuffer path
            kb_buf = sorter.alloc_sort_buffer(dt, n)
            vb_buf = sorter.alloc_sort_buffer("u32", n)
            src = kin.cpu().numpy().view(np.uint32)
            vals = np.arange(n, dtype=np.uint32)

            def pairs_step():
                kb_buf.copy_from_slice(src)
                vb_buf.copy_from_slice(vals)
                sorter.sort_pairs_buffer(kb_buf, vb_buf)
            # device part only: keys/values resident, sort in place each rep
            kd, vd = kin.clone(), torch.arange(n, dtype=torch.int32, device=dev)
            kw, vw = torch.empty_like(kd), torch.empty_like(vd)

            def dev_pairs():
                kw.copy_(kd)
                vw.copy_(vd)
                sorter.sort_pairs_device(dt, kw.data_ptr(), vw.data_ptr(), n, sync=False)
            copy_ms = timed(lambda: (kw.copy_(kd), vw.copy_(vd)), reps)
            ms = timed(dev_pairs, reps) - copy_ms
            t0 = time.perf_counter()
            pairs_step()
            row["sort_buffer_ms"] = round((time.perf_counter() - t0) * 1e3, 3)
            # the buffers untouched by the host since: a sort stays in HBM
            rs = []
            for _ in range(5):
                t0 = time.perf_counter()
                sorter.sort_pairs_buffer(kb_buf, vb_buf)
                rs.append(time.perf_counter() - t0)
            rs.sort()
            row["sort_buffer_again_ms"] = round(rs[len(rs) // 2] * 1e3, 3)
            t0 = time.perf_counter()
            kb_buf.as_slice()
            vb_buf.as_slice()
            row["host_read_back_ms"] = round((time.perf_counter() - t0) * 1e3, 3)
            kb_buf.free()
            vb_buf.free()
        row.update({"ms": round(ms, 4), "mkeys_s": round(n / (ms * 1e-3) / 1e6, 1),
                    "alg_bytes_per_key": bpk,
                    "hbm_frac": round(n * bpk / (ms * 1e-3) / 1e9 / peak, 4), "peak_kind": peak_kind})
        if op == "keys" and n <= (1 << 24):  # the host-slice call, as the reference times it
            h = host if host is not None else kin.cpu().numpy().view(orc.NP_DTYPE[dt])
            hs = [np.array(h, copy=True) for _ in range(5)]
            getattr(sorter, f"sort_{dt}")(np.array(h, copy=True))
            t0 = time.perf_counter()
            for a in hs:
                getattr(sorter, f"sort_{dt}")(a)
            hms = (time.perf_counter() - t0) / len(hs) * 1e3
            row["host_slice"] = {"ms": round(hms, 3), "mkeys_s": round(n / (hms * 1e-3) / 1e6, 1)}
        print(json.dumps(row), flush=True)
        del kin
        torch.cuda.empty_cache()
    sorter.close()


def main():
    args = parse()
    if args.suite:
        run_suite(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
