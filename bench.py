"""Benchmark of the HELLO pricing scan on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--cost l2sq] [--n 1048576] [--d 256] [--k 8] [--precision fp32]

Workload (default): config 5 of the baseline, the isolated pricing scan with
m = n = 1,048,576 points, d = 256, ℓ2² cost, top-k = 8 per row and column;
points ~ N(0, I) fp32, duals f, g ~ N(0, 1) x the median pairwise cost
(estimated from 65,536 sampled pairs, seed 42).  Synthetic data stands in
for the reference's public benchmark features, which are not available here.

A step is one full bidirectional scan: both top-k directions, the five
certificate sums and candidate extraction to device buffers.  `value` is
m*n / (device time per step), inputs resident in HBM, timed with CUDA events
between barriers (max over ranks).  `e2e` runs the host-facing API
(raw_lowrank_bidir_feasibility_pricing_scan) from pinned host arrays with the
uploads and the candidate read-back inside the timed region.  The clouds are
2 GB, larger than L2, so no flush is needed between steps.

With --gpus N (launched under torchrun) source rows are split across ranks
(strong scaling: total work fixed); the target cloud is broadcast once and the
target duals every step, column lists are all-gathered and merged over NCCL.

--impl reference times the reference's own CPU scan (its C++ dot_tile kernel,
built from its sources into oracle/_ref, driven like cpp_violation_scan) on a
bounded row sample of the same workload on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per pair of the scan kernel from an ncu capture of the full
# config-5 launch (dram__bytes_read.sum + dram__bytes_write.sum over its 2^40 pairs), scaled by
# the pairs of the launch; keyed by (d, precision, mode, exact lists)
DRAM_BYTES_PER_PAIR = {(256, "fp32", "one-pass", False): 1.1672, (256, "fp32", "one-pass", True): 1.2835}


# per-path default sizes: config 5 (m = n = 2^20, d = 256) for the l2sq scans, pair costs and
# the PDHG; config 3 (n = m = 262144, d = 128) for the l1 scan
PATH_SIZES = {"scan": (1_048_576, 256), "initial": (1_048_576, 256), "pairs": (1_048_576, 256),
              "pdlp": (1_048_576, 256), "norm": (262_144, 128), "support": (1_048_576, 256),
              "prune": (1_048_576, 256), "coarsest": (1024, 32), "solve": (0, 0)}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--path", default="scan", choices=["scan", "norm", "pairs", "pdlp", "initial", "support", "prune",
                                                   "coarsest", "solve"],
                   help="scan (default, the headline): l2sq pricing scan; norm: l1 scan (config 3 shape); "
                        "pairs: active-support pair costs; pdlp: restricted-OT PDHG iterations; "
                        "initial: l2sq directional top-16 scan (config 5 shape); "
                        "support: active-support candidate filter; prune: budgeted pruning selection; "
                        "coarsest: dense exact transport of a coarsest level (n = m = 1024, d = 32); "
                        "solve: end-to-end hello_ot.solve through the plug-in (--config)")
    p.add_argument("--config", default="C2", choices=sorted(SOLVE_CONFIGS), help="configuration of --path solve")
    p.add_argument("--cost", default="l2sq", choices=["l2sq"])
    p.add_argument("--norm-kind", default="l1", choices=["l1", "linf", "l2"], help="cost of --path norm")
    p.add_argument("--n", type=int, default=None, help="points per side (default: the path's config)")
    p.add_argument("--d", type=int, default=None, help="feature dimension (default: the path's config)")
    p.add_argument("--k", type=int, default=8)
    p.add_argument("--precision", default="fp32", choices=["fp32", "tf32"])
    p.add_argument("--exact", type=int, choices=[0, 1], default=1,
                   help="1 (default): the fp64 re-check of the l2sq lists (HB_L2SQ_EXACT); 0: fp32-class lists")
    p.add_argument("--passes", type=int, choices=[1, 2], default=None,
                   help="force a one-pass (k <= 8) or two-pass scan (default: the library's choice)")
    p.add_argument("--ctas", type=int, choices=[1, 2], default=None,
                   help="one-pass l2sq kernel: 2 = CTA pairs, 1 = single CTAs (default: the library's choice)")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="target length of the CPU baseline sample")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-rows", action="store_true",
                   help="scan path at N = 1: skip the pair-cost and PDHG lines the headline line carries")
    args = p.parse_args()
    n0, d0 = PATH_SIZES[args.path]
    args.n = n0 if args.n is None else args.n
    args.d = d0 if args.d is None else args.d
    return args


def load_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


# ------------------------------------------------------------------ workload
def make_workload(n, d, seed, device, rows=None):
    """Points ~ N(0, I), duals ~ N(0, 1) * median pairwise ℓ2² cost.  `rows`
    (start, stop) limits the source cloud to a block (same values as the full
    cloud's rows).  Generated on `device` with torch's Philox generator."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    y = torch.randn(n, d, device=device, generator=g)
    x_full_seed = seed + 1
    gx = torch.Generator(device=device)
    gx.manual_seed(x_full_seed)
    lo, hi = rows if rows is not None else (0, n)
    # generate the source cloud in fixed 65536-row chunks so a block equals the full cloud's
    # rows, written in place (config 4's clouds are 42 GB each: no concatenated copies)
    chunk = 65536
    x = torch.empty(hi - lo, d, device=device)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        gc = torch.Generator(device=device)
        gc.manual_seed(x_full_seed * 1_000_003 + c0)
        if c1 <= lo or c0 >= hi:
            continue
        block = torch.randn(c1 - c0, d, device=device, generator=gc)
        s0, s1 = max(lo, c0), min(hi, c1)
        x[s0 - lo:s1 - lo] = block[s0 - c0:s1 - c0]
        del block

    def sq_norms(v):  # row norms in fp64, a chunk of rows at a time
        out = torch.empty(v.shape[0], dtype=torch.float64, device=device)
        for r0 in range(0, v.shape[0], chunk):
            out[r0:r0 + chunk] = (v[r0:r0 + chunk].double() ** 2).sum(1)
        return out

    a = sq_norms(x)
    b = sq_norms(y)
    # median pairwise cost from 65536 sampled pairs (seed 42)
    gs = torch.Generator(device=device)
    gs.manual_seed(42)
    si = torch.randint(0, x.shape[0], (65536,), device=device, generator=gs)
    sj = torch.randint(0, n, (65536,), device=device, generator=gs)
    costs = torch.cat([((x[si[c:c + 4096]].double() - y[sj[c:c + 4096]].double()) ** 2).sum(1)
                       for c in range(0, si.numel(), 4096)])
    med = float(costs.median().item())
    f = torch.randn(x.shape[0], device=device, dtype=torch.float64, generator=gs) * med
    gd = torch.randn(n, device=device, dtype=torch.float64, generator=gs) * med
    return x, y, a, b, f, gd, med


SOLVE_CONFIGS = {"C1": (2048, 32, "l2^2"), "C2": (32768, 3, "l2"), "C3": (262144, 128, "l1")}


def solve_config(name, seed=42, n=None):
    """Inputs of the baseline's end-to-end configurations, numpy fp32 points and fp64
    masses (None = uniform): C1 Brenier map (x ~ N(0, I), y = x + 2 tanh(x) row-permuted,
    the reference's examples/quickstart.py), C2 x ~ U[0,1]^3, y ~ U[0,1]^3 + 0.1 N(0, I),
    masses U(0.5, 1.5) normalised, C3 independent 16-component Gaussian mixtures
    (means N(0, 4I), per-component std U(0.5, 1.5), equal weights).  Returns
    (x, y, source_mass, target_mass, cost)."""
    n0, d, cost = SOLVE_CONFIGS[name]
    n = n0 if n is None else int(n)
    rng = np.random.default_rng(seed)
    if name == "C1":
        x = rng.normal(size=(n, d)).astype(np.float32)
        y = x + 2 * np.tanh(x)
        return x, y[rng.permutation(n)], None, None, cost
    if name == "C2":
        x = rng.uniform(size=(n, d)).astype(np.float32)
        y = (rng.uniform(size=(n, d)) + 0.1 * rng.normal(size=(n, d))).astype(np.float32)
        a, b = rng.uniform(0.5, 1.5, n), rng.uniform(0.5, 1.5, n)
        return x, y, a / a.sum(), b / b.sum(), cost

    def mixture():
        means = rng.normal(scale=2.0, size=(16, d))
        stds = rng.uniform(0.5, 1.5, 16)
        comp = rng.integers(0, 16, n)
        return (means[comp] + stds[comp, None] * rng.normal(size=(n, d))).astype(np.float32)

    x = mixture()
    return x, mixture(), None, None, cost


# ------------------------------------------------------------------ clocks
class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.path = Path(tempfile.mkstemp(prefix="clocks", suffix=".csv")[1])
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in self.path.read_text().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ reference CPU scan
def reference_cpu_scan(x, y, a, b, f, g, k, scale, threads):
    """The reference's CPU ℓ2² scan: torch.mm product tiles and its C++ dot_tile
    kernel (src/hello_ot/kernels/cpp_scan.py:95-182, _native/cpp/scan.cpp:137-227),
    with the tile shape of torch_scan._tile_shape (64 MB budget)."""
    import oracle

    ext = oracle.load_ref("scan")
    ns, m = x.shape[0], y.shape[0]
    rk, ck = min(k, m), min(k, ns)
    rv = torch.full((ns, rk), -torch.inf, dtype=torch.float64)
    ri = torch.full((ns, rk), -1, dtype=torch.int64)
    cv = torch.full((m, ck), -torch.inf, dtype=torch.float64)
    ci = torch.full((m, ck), -1, dtype=torch.int64)
    sb = min(ns, 256)
    tb = min(m, max(1, (64 * 1024 * 1024 // 32) // sb))
    stats = [0.0, 0.0, 0, 0.0, 0.0]
    for s0 in range(0, ns, sb):
        s1 = min(ns, s0 + sb)
        for t0 in range(0, m, tb):
            t1 = min(m, t0 + tb)
            prod = torch.mm(x[s0:s1], y[t0:t1].T)
            num, den, cnt, mx, cm = ext.dot_tile(prod.numpy(), a[s0:s1].numpy(), b[t0:t1].numpy(),
                                                 f[s0:s1].numpy(), g[t0:t1].numpy(), rv[s0:s1].numpy(),
                                                 ri[s0:s1].numpy(), cv[t0:t1].numpy(), ci[t0:t1].numpy(), scale,
                                                 s0, t0, 0, threads)
            stats[0] += num; stats[1] += den; stats[2] += cnt
            stats[3] = max(stats[3], mx); stats[4] = max(stats[4], cm)
    rm, cmk = rv > 0, cv > 0
    rows = torch.cat((torch.arange(ns)[:, None].expand(-1, rk)[rm], ci[cmk]))
    return rows.numel(), stats


def reference_scan_sample(args, steps, warmup):
    """Seconds per step of the reference's CPU scan over a bounded row sample of the
    configured workload (same seed and distribution as the device clouds, generated on
    the host), sized so one step takes about cpu_seconds / 2.  Both the reference arm
    and the repo arm's cpu_baseline leg time the scan through this function, the repo
    arm before any GPU work, so the two figures measure the same thing."""
    import oracle

    oracle.load_ref("scan")  # raises when the reference's CPU build is missing
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n, d, k = args.n, args.d, args.k
    x, y, a, b, f, g, _ = make_workload(n, d, 42, torch.device("cpu"), rows=(0, 16384))
    probe = 64
    t0 = time.perf_counter()
    reference_cpu_scan(x[:probe], y, a[:probe], b, f[:probe], g, k, 2.0, threads)
    dt = time.perf_counter() - t0
    rows = int(min(x.shape[0], max(probe, probe * (args.cpu_seconds / 2) / max(dt, 1e-3))))
    rows = max(probe, rows // 64 * 64)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        reference_cpu_scan(x[:rows], y, a[:rows], b, f[:rows], g, k, 2.0, threads)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    sample = (f"{rows} source rows x {n} targets per step (d={d}, k={k}), reference dot_tile (scan.cpp) + "
              f"torch.mm tiles, {warmup} warm-up + {steps} timed step(s)")
    return sec, rows, threads, sample


def other_rows(args):
    """The pair-cost (SDDMM) and PDHG rows at their config-5 sizes, each measured by this
    script's own --path run in a child process (CUDA-event timing as in the headline), so
    the headline line carries them too."""
    import subprocess
    rows = {}
    for path in ("pairs", "pdlp"):
        cmd = [sys.executable, str(REPO / "bench.py"), "--path", path, "--steps", str(max(args.steps, 1)),
               "--warmup", str(max(args.warmup, 1)), "--no-cpu"]
        try:
            res = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
            line = json.loads([ln for ln in res.stdout.splitlines() if ln.startswith("{")][-1])
            roof = line.get("roofline", {})
            rows[path] = {"metric": line["metric"], "value": line["value"], "unit": line["unit"],
                          "workload": line["config"]["workload"], "kernel": roof.get("kernel"),
                          "achieved_gbs": roof.get("achieved"), "frac": roof.get("frac"),
                          "iteration_us": roof.get("iteration_us")}
        except Exception as exc:  # report, do not fail the headline
            rows[path] = {"unavailable": str(exc)[:200]}
    return rows


def reference_arm_baseline(args):
    """The repo arm's cpu_baseline: the reference arm itself (`--impl reference` with this run's
    workload, warm-up and step counts) in a child process started before any GPU work, so the
    two figures come from the same procedure in the same kind of process (timed inside this
    process instead, the same sample ran up to 2.7x slower than in the reference arm's)."""
    import subprocess
    cmd = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", str(args.steps),
           "--warmup", str(args.warmup), "--n", str(args.n), "--d", str(args.d), "--k", str(args.k),
           "--cpu-seconds", str(args.cpu_seconds), "--precision", args.precision, "--exact", str(args.exact)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE")}
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
        line = [ln for ln in res.stdout.splitlines() if ln.startswith("{")][-1]
        ref = json.loads(line)
        if "unavailable" in ref:
            raise RuntimeError(ref["unavailable"])
        cb = dict(ref["cpu_baseline"])
        cb["sample"] += "; the reference arm run as a child process before the GPU work"
        return cb
    except Exception as exc:  # reference CPU build missing, or the child failed
        return {"value": None, "unit": "Gpairs/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {exc}"}


# ------------------------------------------------------------------ main arms
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    try:
        sec, rows, threads, sample = reference_scan_sample(args, args.steps, args.warmup)
    except Exception as exc:  # the reference's CPU build is missing
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU backend not built: {exc}"}))
        return
    n = args.n
    value = rows * n / sec / 1e9
    print(json.dumps({
        "impl": "reference", "metric": "pricing-scan Gpairs/s (m·n)", "value": value, "unit": "Gpairs/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32/f64", "data": "synthetic",
        "config": workload_config(args),
        "cpu_baseline": {"value": value, "unit": "Gpairs/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": "Gpairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def scan_mode(args):
    if args.passes is not None:
        return "one-pass" if args.passes == 1 else "two-pass"
    one = args.k <= 8 and (args.d >= 128 or (args.d >= 64 and args.n >= 1 << 19))  # the library's rule
    return "one-pass" if one else "two-pass"


def workload_config(args):
    name = {(1_048_576, 256): "C5", (1_280_000, 8192): "C4"}.get((args.n, args.d), "custom")
    return {"workload": f"{name} isolated pricing scan, l2sq, m=n={args.n}, d={args.d}, k={args.k}",
            "n": args.n, "m": args.n, "d": args.d, "topk": args.k, "cost": "l2sq", "dot_scale": 2.0,
            "precision": {"fp32": "3-term fp16 split (fp32-class dot)", "tf32": "1xTF32"}[args.precision],
            "lists": "exact fp64 top-k (fp64 re-check)" if args.exact else "fp32-class top-k",
            "scan_mode": scan_mode(args),
            "parallelism": f"source-row shards x{args.gpus}",
            "l2_policy": "inputs (2 GB clouds) larger than L2; no flush"}


def run_ours(args):
    import __graft_entry__ as entry

    hb = entry.load_package()
    from hello_ot_b200.sharded import ShardedPricingScan, row_partition

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu_baseline = reference_arm_baseline(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import torch.distributed as dist
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    n, d, k = args.n, args.d, args.k
    lo, hi = row_partition(n, world, rank)
    x, y, a, b, f, g, med = make_workload(n, d, 42, dev, rows=(lo, hi))
    if world > 1:  # the target cloud is replicated from rank 0 (once per solve)
        dist.broadcast(y, 0)
        dist.broadcast(b, 0)
    sharded = ShardedPricingScan(precision=args.precision, passes=args.passes, exact=bool(args.exact),
                                 ctas=args.ctas)
    g_step = g.clone()

    def step():
        if world > 1:
            dist.broadcast(g_step, 0)  # target duals change every scan
        r = sharded.scan(x, y, a, b, f, g_step, k, row_offset=lo)
        return r

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches0 = hb.kernel_launch_count()
    hb.set_kernel_timing(True)
    pass_ms = []  # device time of each scan pass kernel, CUDA events inside the library
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        sharded.time_phases = world > 1  # the exchange's own time, reported beside the total
        start.record()
        for _ in range(args.steps):
            step()
            pass_ms.append(hb.last_kernel_times())
        stop.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        sharded.time_phases = False
    hb.set_kernel_timing(False)
    launches = hb.kernel_launch_count() - launches0
    elapsed = start.elapsed_time(stop) / 1e3
    t = torch.tensor([elapsed], device=dev)
    phases = None
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ph = torch.tensor(list(sharded.last_phase_ms() or (0.0, 0.0)), device=dev)
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
        phases = {"local_scan_ms": float(ph[0]), "exchange_ms": float(ph[1]),
                  "note": "last timed step, max over ranks: the rank's scan, then the certificate all-reduce, "
                          "the column-block all-to-all, merge and all-gather and the candidate gather to rank 0"}
    sec = float(t.item()) / args.steps
    value = n * n / sec / 1e9

    nk = len(pass_ms[0]) if pass_ms else 0
    times = [sum(p[j] for p in pass_ms) / len(pass_ms) for j in range(nk)] \
        if nk and all(len(p) == nk for p in pass_ms) else []
    out = None
    if rank == 0:
        peaks, peak_kind = load_peaks()
        rows_local = hi - lo
        mode = scan_mode(args)
        pass1_ms = times[0] if times else float("nan")
        flops = 2.0 * d * rows_local * n  # algorithmic flops of one launch: one dot product per pair
        achieved = flops / (pass1_ms / 1e3) / 1e12
        peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
        per_pair = DRAM_BYTES_PER_PAIR.get((d, args.precision, mode, bool(args.exact)))
        traffic = per_pair * rows_local * n if per_pair else None
        out = {
            "metric": "pricing-scan Gpairs/s (m·n)", "value": value, "unit": "Gpairs/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16x3/f64" if args.precision == "fp32" else "tf32/f64",
            "data": "synthetic (seeded N(0,I) clouds, Gaussian duals scaled by the median cost)",
            "config": workload_config(args),
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": ("hb::l2sq::scan_kernel (one pass: row and column top-k, certificate)"
                                    if mode == "one-pass" else
                                    "hb::l2sq::scan_kernel (pass 1 of 2: source rows, score terms)"),
                         "pass_ms": times, "peak_source": f"{peak_kind} bf16 dense (sustained)",
                         "note": ("algorithmic flops 2*d per pair; the fp32-class split issues 3 fp16 "
                                  "products per pair (3x the algorithmic tensor work)")},
            "clocks": clocks.summary(),
            "median_pair_cost": med,
        }
        if phases:
            out["phases"] = phases
        if args.exact:
            out["exact_rescans"] = dict(zip(("row_lists", "column_lists"), hb.l2sq_last_rescans()))
    # ---- end to end through the host-facing API (pinned host inputs, candidates back to host)
    if not args.no_e2e:
        xh = x.cpu().pin_memory(); yh = y.cpu().pin_memory()
        ah, bh, fh, gh = (v.cpu().pin_memory() for v in (a, b, f, g))
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e2e_times, h2d, d2h = [], 0, 0
        for i in range(max(1, args.steps) + 1):
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            if world == 1:
                r = hb.raw_lowrank_bidir_feasibility_pricing_scan(xh, yh, ah, bh, fh, gh, topk=k, dot_scale=2.0,
                                                                  compute_precision=args.precision,
                                                                  exact=bool(args.exact))
                h2d = sum(v.numel() * v.element_size() for v in (xh, yh, ah, bh, fh, gh))
                d2h = (r.rows.size + r.cols.size) * 8 + 5 * 8
            else:
                xd, yd = xh.to(dev, non_blocking=True), yh.to(dev, non_blocking=True)
                ad, bd, fd, gd = (v.to(dev, non_blocking=True) for v in (ah, bh, fh, gh))
                r = sharded.scan(xd, yd, ad, bd, fd, gd, k, row_offset=lo)
                h2d = sum(v.numel() * v.element_size() for v in (xh, yh, ah, bh, fh, gh))
                if rank == 0:
                    rows_h, cols_h = r.rows.cpu().numpy(), r.cols.cpu().numpy()
                    d2h = (rows_h.size + cols_h.size) * 8
                s = r.stats.cpu()
                d2h += 5 * 8
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            if i > 0:
                e2e_times.append(time.perf_counter() - t0)
        et = torch.tensor([sum(e2e_times) / len(e2e_times)], device=dev)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        if rank == 0:
            out["e2e"] = {"value": n * n / float(et.item()) / 1e9, "unit": "Gpairs/s",
                          "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                          "api": "raw_lowrank_bidir_feasibility_pricing_scan (host arrays)" if world == 1
                          else "ShardedPricingScan.scan from pinned host blocks"}
    if rank == 0 and cpu_baseline is not None:
        out["cpu_baseline"] = cpu_baseline
    if rank == 0 and world == 1 and not args.no_rows:
        out["other_rows"] = other_rows(args)
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ other rows of the path
def _line(args, metric, value, unit, sec, config, extra):
    out = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "data": "synthetic (seeded)", "config": config}
    out.update(extra)
    print(json.dumps(out))


def _timed(fn, args, dev):
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        fn()
    ev1.record()
    torch.cuda.synchronize(dev)
    return ev0.elapsed_time(ev1) / 1e3 / args.steps


def support_problem(n, m, beta, seed):
    """A feasible restricted-OT support: each source and target gets edges, about
    beta (n + m) edges in all (the reference's support budget factor, 10 by default)."""
    rng = np.random.default_rng(seed)
    e_rand = int(beta * (n + m)) - n - m
    rows = np.concatenate([np.arange(n), rng.integers(0, n, m), rng.integers(0, n, e_rand)])
    cols = np.concatenate([rng.integers(0, m, n), np.arange(m), rng.integers(0, m, e_rand)])
    key = np.unique(rows.astype(np.int64) * m + cols)
    rows, cols = key // m, key % m
    perm = rng.permutation(rows.size)
    cost = rng.random(rows.size) * 4.0
    return rows[perm], cols[perm], cost[perm], np.full(n, 1.0 / n), np.full(m, 1.0 / m)


def run_pdlp(args, hb, dev, peaks):
    """Restricted-OT PDHG: a step is `iters` iterations (evaluation every 200) on a
    support of 10 (n + m) edges; metric iterations/s; roofline HBM bytes/iteration."""
    n = m = args.n
    iters = 1000
    rows, cols, cost, a, b = support_problem(n, m, 10.0, 42)
    e = rows.size
    R, C, W = (torch.as_tensor(v, device=dev) for v in (rows, cols, cost))
    A, B = torch.as_tensor(a, device=dev), torch.as_tensor(b, device=dev)
    solver = hb.NativeRestrictedOTPDLP(device=dev, evaluation_frequency=200, iteration_limit=iters)
    hb.set_kernel_timing(True)
    sec = _timed(lambda: solver.solve_restricted(rows=R, cols=C, costs=W, source_mass=A, target_mass=B, tolerance=0.0),
                 args, dev)
    block_ms = hb.last_kernel_times()
    hb.set_kernel_timing(False)
    per_iter = (block_ms[0] / 200 / 1e3) if block_ms else sec / iters
    # the same solve with atomic node sums (run-to-run summation order; not the default)
    fast = hb.NativeRestrictedOTPDLP(device=dev, evaluation_frequency=200, iteration_limit=iters, deterministic=False)
    hb.set_kernel_timing(True)
    fast_sec = _timed(lambda: fast.solve_restricted(rows=R, cols=C, costs=W, source_mass=A, target_mass=B,
                                                    tolerance=0.0), args, dev)
    fast_ms = hb.last_kernel_times()
    hb.set_kernel_timing(False)
    fast_iter = (fast_ms[0] / 200 / 1e3) if fast_ms else fast_sec / iters
    # algorithmic bytes: one copy of the edge state (x read + write, anchor, scaled cost, both
    # endpoints) and the node state; the fused pass streams the edge state in both orders:
    # per edge and side x, anchor, scaled cost, x write (8 B each), the other endpoint (4 B),
    # the own endpoint's place in its tile (1 B)
    bytes_iter = 44 * e + 32 * (n + m)
    stream_iter = 2 * 37 * e + 64 * (n + m)
    achieved = bytes_iter / per_iter / 1e9
    extra = {"dtype": "f64", "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                                          "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                                          "kernel": "hb::pdlp::fused_pass (one launch per iteration, both sides)",
                                          "bytes_per_iteration": bytes_iter, "iteration_us": per_iter * 1e6,
                                          "streamed_bytes_per_iteration": stream_iter,
                                          "streamed_gbs": stream_iter / per_iter / 1e9},
             "atomic_sums": {"iterations_per_s": iters / fast_sec, "iteration_us": fast_iter * 1e6,
                             "achieved_gbs": bytes_iter / fast_iter / 1e9,
                             "note": "deterministic=False: node sums by atomics in the edge pass"}}
    if not args.no_cpu:
        import oracle
        lp = oracle.load_ref("lp")
        threads = os.cpu_count() or 1
        cpu_iters = 40
        masses = np.concatenate((a, b))
        t0 = time.perf_counter()
        lp.solve_once(rows, cols, cost, masses, np.zeros(e), np.zeros(n + m), n, threads, 200, 3600.0, cpu_iters,
                      0.0, 0.0, 0.0, False, False)
        dt = time.perf_counter() - t0
        extra["cpu_baseline"] = {"value": cpu_iters / dt, "unit": "iterations/s", "cores": threads,
                                 "kind": "reference", "sample": f"{cpu_iters} iterations of the reference C++ "
                                                                 f"solve_once (solver.cpp) on the same support"}
    _line(args, "restricted-OT PDHG iterations/s", iters / sec, "iterations/s", sec,
          {"workload": f"restricted OT, n=m={n}, E={e} (10 (n+m)), {iters} iterations per step", "n": n, "m": m,
           "edges": e}, extra)


def run_pairs(args, hb, dev, peaks):
    """Active-support pair costs: a step evaluates E = 8 (n + m) candidate edges
    (k = 8 per row and column) of an n x n, d-dim problem; metric Gedges/s.  The
    edges come grouped by source row, the order the reference's CSR-blocked
    evaluation uses (pairs.py:380-412); targets are random."""
    n, d = args.n, args.d
    e = 8 * 2 * n
    g = torch.Generator(device=dev)
    g.manual_seed(42)
    x = torch.randn(n, d, device=dev, generator=g)
    y = torch.randn(n, d, device=dev, generator=g)
    a, b = (x.double() ** 2).sum(1), (y.double() ** 2).sum(1)
    rows = torch.sort(torch.randint(0, n, (e,), device=dev, generator=g)).values
    cols = torch.randint(0, n, (e,), device=dev, generator=g)
    hb.set_kernel_timing(True)
    sec = _timed(lambda: hb.pair_costs(3, x, y, rows, cols, a, b, 2.0), args, dev)
    kms = hb.last_kernel_times()
    # the same edges in random order (every source row gathered per edge)
    perm = torch.randperm(e, device=dev, generator=g)
    rows_r, cols_r = rows[perm].contiguous(), cols[perm].contiguous()
    sec_r = _timed(lambda: hb.pair_costs(3, x, y, rows_r, cols_r, a, b, 2.0), args, dev)
    kms_r = hb.last_kernel_times()
    hb.set_kernel_timing(False)
    # algorithmic bytes: indices + output per edge, each source row once, each target row per edge
    # (random targets have no reuse), row norms once per row
    u_r = int(torch.unique(rows).numel())
    bytes_call = e * (8 + 8 + 8 + 4 * d) + u_r * (4 * d + 8) + 8 * int(torch.unique(cols).numel())
    achieved = bytes_call / (kms[0] / 1e3) / 1e9 if kms else bytes_call / sec / 1e9
    extra = {"dtype": "f32 in, f64 accumulate", "roofline": {
        "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": achieved / peaks["hbm_gbs"], "traffic": None,
        "kernel": f"hb::pairs::pair_kernel_ring<3,{d // 128}>" if d in (128, 256, 512) else "hb::pairs::pair_kernel",
        "bytes_per_edge": bytes_call / e,
        "note": "each source row once, each target row per edge (no target reuse on a random support)"},
        "random_order": {"value": e / sec_r / 1e9, "unit": "Gedges/s",
                         "kernel_ms": kms_r[0] if kms_r else None,
                         "gathered_gbs": e * (24 + 8 * d) / (kms_r[0] / 1e3) / 1e9 if kms_r else None}}
    if not args.no_cpu:  # the reference's CPU branch: a[r] + b[c] - s * einsum (pairs.py:296-307)
        xs, ys = x.cpu().numpy(), y.cpu().numpy()
        asub, bsub = a.cpu().numpy().astype(np.float32), b.cpu().numpy().astype(np.float32)
        rs, cs = rows[:200000].cpu().numpy(), cols[:200000].cpu().numpy()
        t0 = time.perf_counter()
        _ = (asub[rs] + bsub[cs]) - 2.0 * np.einsum("nd,nd->n", xs[rs], ys[cs])
        dt = time.perf_counter() - t0
        extra["cpu_baseline"] = {"value": rs.size / dt / 1e9, "unit": "Gedges/s", "cores": 1, "kind": "port",
                                 "sample": f"{rs.size} edges with the reference's numpy CPU branch"}
    _line(args, "pair costs Gedges/s", e / sec / 1e9, "Gedges/s", sec,
          {"workload": f"l2sq pair costs, E={e} edges of a {n} x {n} problem grouped by source row, "
                       f"random targets, d={d}", "edges": e, "d": d}, extra)


def run_norm(args, hb, dev, peaks):
    """Norm pricing scan (ℓ1 by default), config 3 shape (n = m = 262144, d = 128, k = 8)."""
    n, d, k, kind = args.n, args.d, args.k, args.norm_kind
    g = torch.Generator(device=dev)
    g.manual_seed(42)
    x = torch.randn(n, d, device=dev, generator=g)
    y = torch.randn(n, d, device=dev, generator=g)
    # duals ~ N(0, 1) x the median pairwise cost (65536 sampled pairs), as config 5 specifies
    sr = torch.randint(0, n, (65536,), device=dev, generator=g)
    sc = torch.randint(0, n, (65536,), device=dev, generator=g)
    med = float(hb.pair_costs({"l1": 0, "linf": 1, "l2": 2}[kind], x, y, sr, sc).median())
    f = torch.randn(n, device=dev, dtype=torch.float64, generator=g) * med
    gg = torch.randn(n, device=dev, dtype=torch.float64, generator=g) * med
    hb.set_kernel_timing(True)
    sec = _timed(lambda: hb.norm_scan(x, y, f, gg, k, kind), args, dev)
    kms = hb.last_kernel_times()
    hb.set_kernel_timing(False)
    # FP32-pipe roofline: 2 d instructions per pair; peak = 148 SMs x 128 lanes x max clock
    sm, mhz = torch.cuda.get_device_properties(dev).multi_processor_count, peaks.get("sm_max_mhz", 1965.0)
    peak = sm * 128 * mhz * 1e6 / 1e12
    achieved = 2 * d * n * n / (kms[0] / 1e3) / 1e12 if kms else float("nan")
    extra = {"dtype": "f32 distance, f64 score", "roofline": {
        "bound": "fp32 pipe", "achieved": achieved, "peak": peak, "unit": "Tinst/s", "frac": achieved / peak,
        "traffic": None, "kernel": f"hb::norm::scan_kernel ({kind}; one pass: row and column lists)",
        "peak_source": "nominal: SMs x 128 fp32 lanes x max SM clock"}}
    if not args.no_cpu:
        import oracle
        rows = 64
        xs, ys = x[:rows].cpu().numpy(), y.cpu().numpy()
        t0 = time.perf_counter()
        oracle.scan(kind, xs, ys, f[:rows].cpu().numpy(), gg.cpu().numpy(), rk=k, ck=0, exact=False,
                    threads=os.cpu_count() or 1)
        dt = time.perf_counter() - t0
        extra["cpu_baseline"] = {"value": rows * n / dt / 1e9, "unit": "Gpairs/s", "cores": os.cpu_count() or 1,
                                 "kind": "port", "sample": f"{rows} source rows x {n} targets, oracle fp32 model"}
    _line(args, f"{kind} pricing-scan Gpairs/s (m·n)", n * n / sec / 1e9, "Gpairs/s", sec,
          {"workload": f"{kind} pricing scan, n=m={n}, d={d}, k={k}", "n": n, "d": d, "topk": k,
           "median_pair_cost": med}, extra)


def run_initial(args, hb, dev, peaks):
    """ℓ2² directional (initial) scan: each source row's best kappa = 16 of (2<x,y> - a) + (g - b),
    config 5 shape (m = n = 1,048,576, d = 256) unless --n/--d say otherwise."""
    n, d, k = args.n, args.d, 16
    x, y, a, b, f, g, med = make_workload(n, d, 42, dev, rows=(0, n))
    qb, dbb = -a, g - b
    hb.set_kernel_timing(True)
    sec = _timed(lambda: hb.l2sq_topk(x, y, qb, dbb, k, dot_scale=2.0, precision=args.precision), args, dev)
    kms = hb.last_kernel_times()
    hb.set_kernel_timing(False)
    peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
    achieved = 2.0 * d * n * n / (kms[0] / 1e3) / 1e12 if kms else float("nan")
    extra = {"dtype": "f16x3/f64" if args.precision == "fp32" else "tf32/f64", "roofline": {
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
        "traffic": None, "kernel": "hb::l2sq::scan_kernel<16, 0, 0, 0> (row lists only)",
        "peak_source": "measured bf16 dense (sustained)",
        "note": "algorithmic flops 2*d per pair; the fp32-class split issues 3 fp16 products per pair"}}
    if not args.no_cpu:  # the reference's CPU directional scan is torch tiles + topk; the oracle port stands in
        import oracle
        rows = 32
        xs, ys = x[:rows].cpu().numpy(), y.cpu().numpy()
        t0 = time.perf_counter()
        oracle.scan("raw", xs, ys, qb[:rows].cpu().numpy(), dbb.cpu().numpy(), a[:rows].cpu().numpy(),
                    b.cpu().numpy(), dot_scale=2.0, rk=k, ck=0, threads=os.cpu_count() or 1)
        dt = time.perf_counter() - t0
        extra["cpu_baseline"] = {"value": rows * n / dt / 1e9, "unit": "Gpairs/s", "cores": os.cpu_count() or 1,
                                 "kind": "port", "sample": f"{rows} source rows x {n} targets in {dt:.1f} s, "
                                                           "oracle fp64 row scan"}
    _line(args, "l2sq initial directional scan Gpairs/s (m·n)", n * n / sec / 1e9, "Gpairs/s", sec,
          {"workload": f"l2sq directional top-{k} scan, n=m={n}, d={d}", "n": n, "d": d, "topk": k,
           "median_pair_cost": med}, extra)


def run_support(args, hb, dev, peaks):
    """Active-support filter (ActiveSupport.filter_new_candidate_pairs): a support of
    10 (n + m) unsorted keys and the 8 (n + m) row-side plus 8 (n + m) column-side
    candidates of one scan, a third of them already in the support; metric candidates/s."""
    n = m = args.n
    g = torch.Generator(device=dev)
    g.manual_seed(42)
    size, cand = 10 * (n + m), 16 * (n + m)
    keys = torch.unique(torch.randint(0, n * m, (int(size * 1.05),), device=dev, generator=g))[:size]
    keys = keys[torch.randperm(keys.numel(), device=dev, generator=g)]
    old = keys[torch.randint(0, keys.numel(), (cand // 3,), device=dev, generator=g)]
    ck = torch.cat([old, torch.randint(0, n * m, (cand - old.numel(),), device=dev, generator=g)])
    rows, cols = (ck // m).to(torch.int32), (ck % m).to(torch.int32)
    hb.set_kernel_timing(True)
    sec = _timed(lambda: hb.filter_new_candidate_pairs(keys, n, m, rows, cols), args, dev)
    hb.set_kernel_timing(False)
    new = hb.filter_new_candidate_pairs(keys, n, m, rows, cols)[3]
    bytes_call = 8 * cand + 8 * keys.numel() + 8 * new  # read candidates and support keys, write new pairs
    achieved = bytes_call / sec / 1e9
    extra = {"dtype": "int64 keys", "roofline": {
        "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": achieved / peaks["hbm_gbs"], "traffic": None,
        "kernel": "hb::support (CUB radix sorts of both key sets, flag pass, compaction)",
        "note": "algorithmic bytes: candidates and support keys read once, new pairs written once; "
                "the radix sorts move each key several times"}}
    if not args.no_cpu:  # the reference's own torch calls (active_support.py:483-506) on the host, 1/16 sample
        kc, rc_, cc_ = keys[: keys.numel() // 16].cpu(), rows[: cand // 16].cpu(), cols[: cand // 16].cpu()
        t0 = time.perf_counter()
        ck2 = torch.unique(rc_.to(torch.int64) * m + cc_.to(torch.int64), sorted=True)
        act = torch.sort(kc).values
        pos = torch.searchsorted(act, ck2)
        mem = (pos < act.numel()) & (act[pos.clamp_max(act.numel() - 1)] == ck2)
        _ = ck2[~mem]
        dt = time.perf_counter() - t0
        extra["cpu_baseline"] = {"value": rc_.numel() / dt / 1e9, "unit": "Gcandidates/s",
                                 "cores": torch.get_num_threads(), "kind": "port",
                                 "sample": f"{rc_.numel()} candidates against {kc.numel()} support keys, "
                                           "the reference's torch calls on the host"}
    _line(args, "support filter Gcandidates/s", cand / sec / 1e9, "Gcandidates/s", sec,
          {"workload": f"support filter, n=m={n}, support {keys.numel()} keys, {cand} candidates",
           "n": n, "m": m, "support": int(keys.numel()), "candidates": cand, "new": int(new)}, extra)


def run_prune(args, hb, dev, peaks):
    """Budgeted pruning selection (DualGapCleaning, protect-new): a support of 10 (n + m)
    edges, 30% with flow, creation iterations spread over the last few; remove the 20%
    with the largest reduced costs among the old zero-flow edges; metric edges/s."""
    n = m = args.n
    e = 10 * (n + m)
    g = torch.Generator(device=dev)
    g.manual_seed(42)
    rows = torch.randint(0, n, (e,), device=dev, generator=g, dtype=torch.int32)
    cols = torch.randint(0, m, (e,), device=dev, generator=g, dtype=torch.int32)
    costs = torch.rand(e, device=dev, generator=g, dtype=torch.float64) * 3
    x = torch.where(torch.rand(e, device=dev, generator=g) < 0.3,
                    torch.rand(e, device=dev, generator=g, dtype=torch.float64), torch.zeros((), device=dev,
                                                                                           dtype=torch.float64))
    creation = torch.randint(-2, 6, (e,), device=dev, generator=g, dtype=torch.int32)
    duals = torch.randn(n + m, device=dev, generator=g, dtype=torch.float64)
    num = e // 5
    sec = _timed(lambda: hb.select_prune_positions(rows, cols, costs, x, creation, duals, n, m, num, 5), args, dev)
    bytes_call = e * (4 + 4 + 8 + 8 + 4) + 4 * num  # edge arrays read once, positions written
    achieved = bytes_call / sec / 1e9
    extra = {"dtype": "f64 reduced costs, int32 positions", "roofline": {
        "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": achieved / peaks["hbm_gbs"], "traffic": None,
        "kernel": "hb::support prune (values pass, compaction, stable radix sort of the removable edges)",
        "note": "algorithmic bytes: the five edge arrays read once, positions written once; the sort moves "
                "the removable edges' keys several times"}}
    if not args.no_cpu:  # the reference's torch calls (pruning_values + _select_zero_flow_removals), 1/16 sample
        k = e // 16
        r_, c_, w_, x_, cr_ = (t[:k].cpu() for t in (rows, cols, costs, x, creation))
        d_ = duals.cpu()
        t0 = time.perf_counter()
        rc = w_ - (d_[:n].index_select(0, r_.long()) + d_[n:].index_select(0, c_.long()))
        rc = torch.where(torch.isfinite(rc), rc, torch.full_like(rc, -torch.inf))
        pool = (cr_ != 5) & (cr_ != -1) & ~(x_.abs() > 1e-15)
        idx = torch.nonzero(pool, as_tuple=False).view(-1)
        order = torch.argsort(rc.index_select(0, idx), descending=True, stable=True)
        _ = idx.index_select(0, order)[: num // 16]
        dt = time.perf_counter() - t0
        extra["cpu_baseline"] = {"value": k / dt / 1e9, "unit": "Gedges/s", "cores": torch.get_num_threads(),
                                 "kind": "port", "sample": f"{k} edges, the reference's torch calls on the host"}
    _line(args, "pruning selection Gedges/s", e / sec / 1e9, "Gedges/s", sec,
          {"workload": f"budgeted pruning selection, n=m={n}, support {e} edges, remove {num}",
           "n": n, "m": m, "edges": e, "remove": num}, extra)


def coarsest_problem(n, d, seed):
    """A coarsest level of config 1's shape: x ~ N(0, I), y = z + 2 tanh(z), uniform
    masses, dense l2sq cost (fp64)."""
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(n, d))
    z = rng.normal(size=(n, d))
    y = z + 2.0 * np.tanh(z)
    cost = (x * x).sum(1)[:, None] + (y * y).sum(1)[None, :] - 2.0 * x @ y.T
    return np.maximum(cost, 0.0), np.full(n, 1.0 / n), np.full(n, 1.0 / n)


def run_coarsest(args, hb, dev, peaks):
    """Coarsest-level exact transport (the POT ot.emd leaf solve of the reference): a step
    is one dense n x n solve to relative KKT 1e-9 with the plan, duals and distance
    returned; metric solves/s.  value: cost resident on the device; e2e: host cost in,
    host plan and duals out."""
    n, d = args.n, args.d
    cost, a, b = coarsest_problem(n, d, 42)
    C, A, B = (torch.as_tensor(v, device=dev) for v in (cost, a, b))
    out = {}

    def dev_step():
        out["r"] = hb.solve_leaf_from_cost(cost=C, source_mass=A, target_mass=B, tolerance=1e-9, device=dev)

    sec = _timed(dev_step, args, dev)
    r = out["r"]
    iters = r["iterations"]
    e2e_sec = None
    if not args.no_e2e:
        e2e_sec = _timed(lambda: hb.solve_leaf_from_cost(cost=cost, source_mass=a, target_mass=b, tolerance=1e-9,
                                                         device=dev), args, dev)
    e = n * n
    bytes_iter = 44 * e + 32 * (2 * n)
    achieved = bytes_iter * iters / sec / 1e9
    extra = {"dtype": "f64", "roofline": {
        "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": achieved / peaks["hbm_gbs"], "traffic": None,
        "kernel": "hb::pdlp iterations on the complete support (whole solve incl. evaluations and restarts)",
        "bytes_per_iteration": bytes_iter, "iterations": iters},
        "objective": r["distance"], "termination": r["termination_reason"]}
    if e2e_sec is not None:
        extra["e2e"] = {"value": 1.0 / e2e_sec, "unit": "solves/s", "h2d_bytes_per_step": 8 * (e + 2 * n),
                        "d2h_bytes_per_step": 16 * len(r["warm_start_state"].x_prev) + 8 * 2 * n}
    if not args.no_cpu:  # the reference's C++ PDHG (solver.cpp) on the same LP; POT is absent here
        import oracle
        lp = oracle.load_ref("lp")
        threads = os.cpu_count() or 1
        rows = np.repeat(np.arange(n), n)
        cols = np.tile(np.arange(n), n)
        t0 = time.perf_counter()
        ref = lp.solve_once(rows, cols, cost.ravel(), np.concatenate((a, b)), np.zeros(e), np.zeros(2 * n), n,
                            threads, 200, 3600.0, 10 ** 7, 1e-9, 1e-9, 1e-9, False, False)
        dt = time.perf_counter() - t0
        extra["cpu_baseline"] = {"value": 1.0 / dt, "unit": "solves/s", "cores": threads, "kind": "reference",
                                 "sample": f"one solve of the same LP by the reference C++ PDHG (solve_once, "
                                           f"{ref['iterations']} iterations, objective {ref['obj_val']:.12g}); "
                                           "the reference's POT network simplex is not installed"}
    _line(args, "coarsest exact solves/s", 1.0 / sec, "solves/s", sec,
          {"workload": f"coarsest level, dense {n} x {n} l2sq OT, d={d}, relative KKT 1e-9",
           "n": n, "d": d, "edges": e}, extra)


def import_reference(cpp=False):
    """The unmodified reference package, pip-installed into baseline/_ref; cpp=True also
    puts its C++ CPU backend (oracle/_ref, built from its sources) on the path and the
    ot.emd stand-in in place of the absent POT."""
    for p in (REPO / "baseline" / "_ref", REPO / "oracle" / "_ref"):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    if cpp:
        from oracle import pot_emd
        pot_emd.install()
    import hello_ot
    return hello_ot


def reference_solve(name, threads):
    """The reference's own end-to-end solve on its C++ CPU backend (backend="cpp")."""
    hello_ot = import_reference(cpp=True)
    from hello_ot.progress import final_metrics

    x, y, a, b, cost = solve_config(name)
    t0 = time.perf_counter()
    r = hello_ot.solve(x, y, source_mass=a, target_mass=b, cost=cost,
                       options=hello_ot.SolverOptions(backend="cpp", num_threads=threads, verbose="off",
                                                      cost_perturbation="off"))
    return time.perf_counter() - t0, r, final_metrics(r)


def run_solve(args, hb, dev, peaks):
    """End-to-end solve to relative KKT 1e-6: the reference's hello_ot.solve(backend="native")
    with this library bound by hello_ot_b200.plugin, host arrays in, host plan and duals out
    (every host-device copy inside the timed region); metric seconds per solve."""
    from hello_ot_b200 import plugin

    hello_ot = import_reference()
    from hello_ot.progress import final_metrics

    plugin.install(hello_ot)
    name = args.config
    x, y, a, b, cost = solve_config(name)
    opts = hello_ot.SolverOptions(backend="native", verbose="off", cost_perturbation="off")
    out = {}

    def step():
        out["r"] = hello_ot.solve(x, y, source_mass=a, target_mass=b, cost=cost, options=opts)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    plugin.routes(reset=True)
    launches0 = hb.kernel_launch_count()
    times = []
    with ClockSampler(dev.index or 0) as clocks:
        for _ in range(args.steps):
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            step()
            torch.cuda.synchronize(dev)
            times.append(time.perf_counter() - t0)
    launches = hb.kernel_launch_count() - launches0
    routes = plugin.routes()
    sec = sum(times) / len(times)
    r = out["r"]
    pfeas, dfeas, gap, kkt = final_metrics(r)
    n, d = x.shape
    h2d = x.nbytes + y.nbytes + (0 if a is None else a.nbytes + b.nbytes)
    d2h = r.solution.values.size * 24 + 8 * (x.shape[0] + y.shape[0])
    extra = {"higher_is_better": False, "scaling": "none (one GPU)",
             "dtype": "f16x3/f64" if cost == "l2^2" else "f32/f64", "objective": r.objective,
             "relative_kkt": kkt, "primal_feasibility": pfeas, "dual_feasibility": dfeas, "gap": gap,
             "refinement_iterations": r.metadata.get("total_refinement_iterations"),
             "gpu_launches": int(launches),
             "routes_per_step": {k: v / args.steps for k, v in sorted(routes.items())},
             "clocks": clocks.summary(),
             "e2e": {"value": sec, "unit": "s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                     "api": "hello_ot.solve(backend='native') with hello_ot_b200.plugin (host numpy in and out)"}}
    if not args.no_cpu and name in ("C1", "C2"):
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        dt, ref, (rp, rd, rg, rk) = reference_solve(name, threads)
        extra["cpu_baseline"] = {"value": dt, "unit": "s", "cores": threads, "kind": "reference",
                                 "sample": f"one full {name} solve by the reference, backend='cpp' (its C++ "
                                           f"CPU backend), objective {ref.objective!r}, relative KKT {rk:.3g}",
                                 "objective_rel_diff": abs(r.objective - ref.objective) / abs(ref.objective)}
    _line(args, "end-to-end solve time to rel-KKT 1e-6", sec, "s", sec,
          {"workload": f"{name}: {cost}, n=m={n}, d={d}, hello_ot.solve native + hello_ot_b200 plug-in, "
                       "cost_perturbation off", "n": n, "m": int(y.shape[0]), "d": d, "cost": cost}, extra)


def run_other(args):
    import __graft_entry__ as entry

    hb = entry.load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, _ = load_peaks()
    {"pairs": run_pairs, "pdlp": run_pdlp, "norm": run_norm, "initial": run_initial,
     "support": run_support, "prune": run_prune, "coarsest": run_coarsest,
     "solve": run_solve}[args.path](args, hb, dev, peaks)


def run_solve_reference(args):
    """--path solve --impl reference: the reference's own solve on its C++ CPU backend."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    times = []
    for i in range(args.warmup + args.steps):
        dt, r, (rp, rd, rg, rk) = reference_solve(args.config, threads)
        if i >= args.warmup:
            times.append(dt)
    sec = sum(times) / len(times)
    x, y, _, _, cost = solve_config(args.config)
    print(json.dumps({
        "impl": "reference", "metric": "end-to-end solve time to rel-KKT 1e-6", "value": sec, "unit": "s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": False, "scaling": "none", "vs_baseline": None, "dtype": "f32/f64", "data": "synthetic",
        "config": {"workload": f"{args.config}: {cost}, n=m={x.shape[0]}, d={x.shape[1]}, hello_ot.solve "
                               "backend='cpp'", "n": x.shape[0], "d": x.shape[1], "cost": cost},
        "objective": r.objective, "relative_kkt": rk,
        "cpu_baseline": {"value": sec, "unit": "s", "cores": threads, "kind": "reference",
                         "sample": f"whole {args.config} solves, reference C++ CPU backend"},
        "e2e": {"value": sec, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def main():
    args = parse_args()
    if args.path == "solve" and args.impl == "reference":
        run_solve_reference(args)
    elif args.path != "scan":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm is defined for the default "
                                                                  "scan path; other paths report cpu_baseline"}))
            return
        run_other(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
