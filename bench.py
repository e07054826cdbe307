#!/usr/bin/env python3
"""Benchmark of the objeta-cuda hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --case q4_0:151936x2048 [--steps K] [--warmup W]
    python bench.py --grouped 256 [--steps K] [--warmup W]
    python bench.py --official 1,16,256 [--experts E] [--steps K] [--warmup W]

`--case` runs one GEMV of the sweep alone (W + K plain launches, rotating
over its weight copies, no graph) and prints its mean launch time; it is the
command the ncu captures are taken on.  `--grouped T` runs the configs[4]
layer's (expert, token) pairs for T tokens (Zipf(1.1) top-8 of 256 Q4_0
experts, H 2048, I 512) on the grouped tensor-core path and on the CUDA-core
pair programs, W + K calls each, and prints both mean call times; it is the
command the grouped kernel's ncu captures are taken on.  `--official T,..`
runs the official DeepSeek routed experts (configs[3] shapes: split FP4
experts, H 4096, I 2048, top-8 of 256 by default; act_quant FP8 activations)
for T tokens: the pairs on block-scaled tensor cores (moe_pairs_official_tc +
combine) against the CUDA-core official launch once per token.

Workload: the block-quant GEMV format/shape sweep,
Q4_0, Q5_0 and IQ3_0 at rows x cols in {4096x4096, 14336x4096, 4096x14336,
151936x2048}, batch 1.  One step is one pass over those 12 GEMVs.  Weights are
fp32 ~ N(0, 0.02^2) from a seeded generator, packed on the GPU by the library's
byte-exact packers; x ~ N(0, 1).  The FP4 E2M1 GEMV at the same shapes is
timed alongside and reported under "cases" (not in the headline value).

Each rank runs the whole sweep on its own GPU (the GEMV needs no exchange:
weak scaling, replicas), so `value` is the aggregate GB/s over all ranks.
Inputs are larger than L2 in aggregate: every case rotates through enough
copies of its packed weights to cover >= 4x the L2 size, so each launch reads
its weights from HBM.

Prints ONE JSON line (rank 0).  `--impl reference` times the reference's CPU
path (the C restatement of gemv_cpu, all host cores) on the same config.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (151936, 2048)]
HEADLINE_FORMATS = [0, 1, 2]          # Q4_0, Q5_0, IQ3_0
EXTRA_FORMATS = [3]                   # DeepSeek FP4 E2M1 (interleaved), reported per case
FMT_NAMES = {0: "q4_0", 1: "q5_0", 2: "iq3_0", 3: "fp4_e2m1"}
BLOCK_BYTES = {0: 18, 1: 22, 2: 14, 3: 17}
METRIC = "quant GEMV HBM GB/s (BASELINE configs[1] sweep: Q4_0/Q5_0/IQ3_0 x 4 shapes, batch 1)"
FALLBACK_HBM_GBS = 6650.0


def algo_bytes(fmt, rows, cols):
    # packed weights + x + y (the reference counts qbytes + 4*cols, quant.rs:282)
    return rows * (cols // 32) * BLOCK_BYTES[fmt] + 4 * cols + 4 * rows


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._proc = None

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return
        t = threading.Thread(target=self._read, daemon=True)
        t.start()

    def _read(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.samples.append(parts)

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "", 1).isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def read_traffic(kernel_key):
    """DRAM bytes (read + write) per launch of `kernel_key` from the committed
    ncu summary profiles/traffic.json, or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            v = json.load(f).get(kernel_key)
    except (OSError, ValueError):
        return None
    return v.get("dram_bytes_per_launch") if isinstance(v, dict) else v


# --------------------------------------------------------------- our arm
def sweep_config(world):
    """The `config` of the bench line, identical in both arms."""
    return {"workload": "configs[1] GEMV sweep, batch 1", "formats": ["q4_0", "q5_0", "iq3_0"],
            "shapes": [f"{r}x{c}" for r, c in SHAPES], "global_batch": 1 * world,
            "parallelism": f"replicas x{world} (no exchange)",
            "l2_defeat": "weights rotated over >= 4x L2 per case (GPU); CPU: matrices far above the LLC",
            "bytes_per_step": sum(algo_bytes(f, r, c) for f in HEADLINE_FORMATS for r, c in SHAPES)}


def cpu_sweep_inputs(seed=1234):
    """The configs[1] sweep for the CPU leg, packed by the oracle's packers
    (the C restatement of quantize_matrix_cpu): a 64-row tile of
    N(0, 0.02^2) weights per case, repeated to the full matrix (packing the
    full 1.3 G weights on the CPU would take longer than the timing), and
    x ~ N(0, 1).  Both CPU legs (the GPU arm's cpu_baseline and --impl
    reference) time these same bytes."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    inputs = []
    for fmt in HEADLINE_FORMATS:
        for rows, cols in SHAPES:
            nb = rows * (cols // 32) * BLOCK_BYTES[fmt]
            m = (rng.standard_normal(64 * cols) * 0.02).astype(np.float32)
            q = np.resize(O.quantize_matrix(fmt, m, 64, cols), nb)
            x = rng.standard_normal(cols).astype(np.float32)
            inputs.append((fmt, rows, cols, q, x))
    return inputs


def time_cpu_sweep(inputs, threads, passes, warmup):
    """Seconds per pass of the oracle's gemv_cpu over the sweep (row-parallel
    over `threads` threads; 1 = the reference's single-threaded loop), after
    `warmup` untimed passes."""
    from oracle import oracle as O
    for _ in range(warmup):
        for f, r, c, q, x in inputs:
            O.gemv(f, q, x, r, c, threads=threads)
    t = time.perf_counter()
    for _ in range(passes):
        for f, r, c, q, x in inputs:
            O.gemv(f, q, x, r, c, threads=threads)
    return (time.perf_counter() - t) / passes


def cpu_legs(steps, warmup):
    """Both CPU figures on the same packed sweep: all host threads (`steps`
    passes after `warmup`) and one thread (one pass after one warm-up, a
    bounded sample of about 5 s)."""
    inputs = cpu_sweep_inputs()
    step_bytes = sum(algo_bytes(f, r, c) for f, r, c, _, _ in inputs)
    threads = os.cpu_count() or 1
    t_all = time_cpu_sweep(inputs, threads, steps, warmup)
    t_one = time_cpu_sweep(inputs, 1, 1, 1)
    return {"value": round(step_bytes / t_all / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"the full configs[1] sweep (12 GEMVs, {step_bytes} bytes) per pass; {steps} passes after "
                      f"{warmup} warm-up on {threads} threads (row-parallel), 1 pass after 1 warm-up on one thread; "
                      "C restatement of gemv_cpu (quant.rs:627-1019), the Rust reference cannot be built here",
            "single_thread": {"value": round(step_bytes / t_one / 1e9, 3), "unit": "GB/s", "cores": 1,
                              "seconds_per_pass": round(t_one, 3)},
            "seconds_per_pass": round(t_all, 4), "passes": steps}


def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    from objeta_b200.quant import gemv_device

    qb = QuantBackend(local)
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    gen = torch.Generator(device=dev).manual_seed(1234 + 17 * rank)

    cases = []  # dict(fmt, rows, cols, copies[list of uint8 tensors], x, y)
    for fmt in HEADLINE_FORMATS + EXTRA_FORMATS:
        for rows, cols in SHAPES:
            shape = QGemvShape.new(QuantFormat(fmt), rows, cols)
            m = torch.randn(rows, cols, device=dev, generator=gen) * 0.02
            q0 = qb.quantize_matrix_device(QuantFormat(fmt), m, shape)
            del m
            nb = q0.numel()
            ncopy = max(2, math.ceil(4 * l2 / nb))
            copies = [q0] + [q0.clone() for _ in range(ncopy - 1)]
            x = torch.randn(cols, device=dev, generator=gen)
            y = torch.empty(rows, device=dev)
            cases.append(dict(fmt=fmt, rows=rows, cols=cols, copies=copies, x=x, y=y,
                              bytes=algo_bytes(fmt, rows, cols)))
    torch.cuda.synchronize()
    headline = [c for c in cases if c["fmt"] in HEADLINE_FORMATS]
    step_bytes = sum(c["bytes"] for c in headline)

    stream = torch.cuda.Stream(device=dev)
    extra = [c for c in cases if c["fmt"] not in HEADLINE_FORMATS]

    def launch_step(phase, clist, evs=None):
        for i, c in enumerate(clist):
            q = c["copies"][phase % len(c["copies"])]
            if evs is not None:
                evs[2 * i].record(stream)
            gemv_device(c["fmt"], q, c["x"], c["y"], c["rows"], c["cols"], stream)
            if evs is not None:
                evs[2 * i + 1].record(stream)

    # warm-up outside capture (sets kernel attributes, error word)
    with torch.cuda.stream(stream):
        launch_step(0, cases)
    torch.cuda.synchronize()

    def build_graphs(clist, events=True):
        period = max(len(c["copies"]) for c in clist)
        gs, es = [], []
        for p in range(period):
            g = torch.cuda.CUDAGraph()
            evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(2 * len(clist))] \
                if events else None
            with torch.cuda.graph(g, stream=stream):
                launch_step(p, clist, evs)
            gs.append(g)
            es.append(evs)
        return gs, es

    def timed(gs, es, clist, steps, warmup, sampler=None):
        period = len(gs)
        for s in range(warmup):
            with torch.cuda.stream(stream):
                gs[s % period].replay()
        torch.cuda.synchronize()
        if sampler is not None:
            sampler.start()
            time.sleep(0.3)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        per = [0.0] * len(clist)
        t0.record(stream)
        for s in range(steps):
            with torch.cuda.stream(stream):
                gs[(warmup + s) % period].replay()
        t1.record(stream)
        torch.cuda.synchronize()
        if sampler is not None:
            sampler.stop()
        # each phase's events hold its last replay; average over phases used
        used = sorted({(warmup + s) % period for s in range(steps)})
        for p in used:
            if es[p] is None:
                continue
            for i in range(len(clist)):
                per[i] += es[p][2 * i].elapsed_time(es[p][2 * i + 1]) / len(used)
        if world > 1:
            dist.barrier()
        return t0.elapsed_time(t1), per

    # The headline times the sweep as a caller runs it: back to back, no
    # instrumentation between the GEMVs.  Per-case times (and the roofline of
    # the dominant case) come from a second set of graphs with an event pair
    # around every GEMV.
    plain, _ = build_graphs(headline, events=False)
    graphs, graph_events = build_graphs(headline)
    xgraphs, xevents = build_graphs(extra)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    elapsed, _ = timed(plain, [None] * len(plain), headline, args.steps, args.warmup, sampler)
    _, per_head = timed(graphs, graph_events, headline, max(3, min(args.steps, 10)), 3)
    _, per_extra = timed(xgraphs, xevents, extra, max(3, min(args.steps, 10)), 3)
    if world > 1:
        t = torch.tensor([elapsed], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    value = step_bytes * args.steps * world / (elapsed / 1e3) / 1e9
    per_case_ms = per_head + per_extra
    cases = headline + extra

    # dominant kernel: the sweep case with the largest share of the step.  Its
    # average launch duration is measured on its own: a graph of 8 back-to-back
    # launches (rotating weight copies) replayed, CUDA events around the
    # replays on the launching stream; one launch = the GEMV's two kernels,
    # the x-image prep and the pipelined GEMV.
    dom = max(range(len(headline)), key=lambda i: per_case_ms[i])
    dc = headline[dom]
    peak, peak_kind = read_peaks()
    per_launch_ms = dominant_launch_ms(dc, stream, max(10, args.steps), args.warmup)
    achieved = dc["bytes"] / (per_launch_ms / 1e3) / 1e9
    dom_name = f"{FMT_NAMES[dc['fmt']]}_{dc['rows']}x{dc['cols']}"
    roofline = {"bound": "hbm",
                "kernel": ("" if gemv_launches(dc["cols"]) == 1 else "ximage + ") +
                          f"pipe_kernel<RowDot<{FMT_NAMES[dc['fmt']]}>> GEMV {dc['rows']}x{dc['cols']}",
                "achieved": round(achieved, 1), "peak": peak, "peak_source": f"{peak_kind} (hbm_gbs)",
                "unit": "GB/s", "frac": round(achieved / peak, 4),
                "algorithmic_bytes_per_launch": dc["bytes"],
                "us_per_launch": round(per_launch_ms * 1e3, 2),
                "us_per_launch_in_sweep": round(per_case_ms[dom] * 1e3, 2),
                "traffic": read_traffic(f"gemv_{dom_name}")}
    case_out = {}
    for i, c in enumerate(cases):
        gbs = c["bytes"] / (per_case_ms[i] / 1e3) / 1e9
        case_out[f"{FMT_NAMES[c['fmt']]}_{c['rows']}x{c['cols']}"] = {
            "us": round(per_case_ms[i] * 1e3, 2), "GB/s": round(gbs, 1),
            "frac_of_peak": round(gbs / peak, 4)}

    # ---- e2e through the public host-slice API (QuantBackend.gemv)
    e2e = run_e2e(qb, cases, headline, args, world, rank, dev)

    # ---- MoE configs (reported beside the headline)
    moe = {}
    if not args.no_moe:
        for c in cases:
            c["copies"] = c["copies"][:1]
        torch.cuda.empty_cache()
        msteps = max(3, min(args.steps, 20))
        moe["c3_q4_stack"] = bench_c3(qb, dev, gen, msteps, args.warmup, peak)
        moe["c4_fp4_shared"] = bench_c4(dev, gen, msteps, args.warmup, peak)
        moe["c5_ep_resident"] = bench_c5_resident(qb, dev, gen, world, rank, None, msteps, args.warmup, peak)
        moe["c5_ep_cache"] = bench_c5_cache(qb, dev, gen, world, rank, None, msteps, args.warmup, peak)

    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "u4/u5/u3 codes x int digits of x (21-bit per-block fixed point; outlier blocks in f32): "
                     "exact int32 block sums, f16 scales, f32 accumulate",
            "data": "synthetic: weights ~N(0,0.02^2) packed on device, x ~N(0,1), seeded",
            "config": sweep_config(world),
            "timing": "headline: CUDA-graph replays of the 12 GEMVs back to back; per case: event pairs",
            "roofline": roofline, "cases": case_out, "e2e": e2e, "moe": moe,
            "gpu_launches": args.steps * sum(gemv_launches(c["cols"]) for c in headline),
            "clocks": sampler.summary(),
        }
        result["cpu_baseline"] = cpu_legs(max(3, min(args.steps, 10)), 2)
        if "c5_ep_resident" in moe:
            result["ep"] = ep_summary(moe["c5_ep_resident"], world)
        # last, so that a reader keeping only the line's tail keeps it: every
        # case's fraction of peak and the MoE configs in a few numbers
        result["summary"] = line_summary(case_out, moe, result.get("ep"), result["cpu_baseline"])
    if world > 1:
        dist.barrier()
        del graphs, xgraphs, plain
        dist.destroy_process_group()
    return result


def line_summary(case_out, moe, ep, cpu):
    """A compact digest of the line (under ~1.2 KB)."""
    out = {"case_frac_of_peak": {k: v["frac_of_peak"] for k, v in case_out.items()}}
    for key, name in (("c3_q4_stack", "c3"), ("c4_fp4_shared", "c4")):
        if key in moe:
            out[name] = {"us_per_token": moe[key]["us_per_token"], "frac": moe[key]["frac_of_hbm"]}
    if ep:
        out["c5_resident"] = {k: {"tok_s": v["tokens_per_s"], "frac": v["frac_of_aggregate_hbm"],
                                  "largest_phase": v.get("largest_phase")}
                              for k, v in ep.items() if k.startswith("T")}
    if "c5_ep_cache" in moe:
        out["c5_cache_pcie_GBs"] = {k: v["pcie_GB/s_all_ranks"] for k, v in moe["c5_ep_cache"].items()
                                    if k.startswith("T")}
        out["c5_cache_frac_of_h2d"] = {k: v["pcie_frac_of_measured_h2d"] for k, v in moe["c5_ep_cache"].items()
                                       if k.startswith("T")}
    out["cpu_GBs"] = {"threads": cpu["value"], "one_thread": cpu["single_thread"]["value"]}
    return out


def gemv_launches(cols):
    """Kernels one digit-format GEMV launches (x 16-byte aligned): the
    pipelined kernel alone up to 4096 columns, where it builds the x image
    itself, else an x-image launch before it."""
    return 1 if cols <= 4096 else 2


def dominant_launch_ms(c, stream, steps, warmup):
    """Average device time of one launch of sweep case `c` in steady state:
    a CUDA graph of 8 launches over rotating weight copies, replayed."""
    import torch
    from objeta_b200.quant import gemv_device
    n = 8
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n):
            gemv_device(c["fmt"], c["copies"][i % len(c["copies"])], c["x"], c["y"], c["rows"], c["cols"], stream)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        with torch.cuda.stream(stream):
            g.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    del g
    return t0.elapsed_time(t1) / (steps * n)


def run_e2e(qb, cases, headline, args, world, rank, dev):
    """Same metric through QuantBackend.gemv: host (pinned) weights and x in,
    host y out, H2D + kernel + D2H per call, like the reference API."""
    import torch
    import torch.distributed as dist
    from objeta_b200 import QGemvShape, QuantFormat
    from objeta_b200._lib import call
    hosts = []
    for c in headline:
        w = c["copies"][0].cpu().numpy()
        x = c["x"].cpu().numpy()
        call("objb_host_register", w.ctypes.data, w.nbytes)
        call("objb_host_register", x.ctypes.data, x.nbytes)
        hosts.append((c, w, x))
    steps = max(1, min(args.steps, 3))
    # one untimed pass
    for c, w, x in hosts:
        qb.gemv(QuantFormat(c["fmt"]), None, w, x, QGemvShape.new(QuantFormat(c["fmt"]), c["rows"], c["cols"]))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t = time.perf_counter()
    h2d = d2h = 0
    for _ in range(steps):
        for c, w, x in hosts:
            y, _tel = qb.gemv(QuantFormat(c["fmt"]), None, w, x,
                              QGemvShape.new(QuantFormat(c["fmt"]), c["rows"], c["cols"]))
            h2d += w.nbytes + x.nbytes
            d2h += y.nbytes
    el = time.perf_counter() - t
    if world > 1:
        tt = torch.tensor([el], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        el = float(tt.item())
    for c, w, x in hosts:
        call("objb_host_unregister", w.ctypes.data)
        call("objb_host_unregister", x.ctypes.data)
    step_bytes = sum(c["bytes"] for c in headline)
    return {"value": round(step_bytes * steps * world / el / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d // steps, "d2h_bytes_per_step": d2h // steps,
            "steps": steps, "api": "QuantBackend.gemv (objb_gemv_host): H2D weights+x, kernel, D2H y per call",
            "timer": "host wall clock (perf_counter), each call synchronous like the reference"}


# ------------------------------------------------------------ MoE configs
C3 = dict(layers=4, experts=8, top_k=2, hidden=4096, inter=14336)
C4 = dict(experts=256, top_k=8, hidden=4096, inter=2048)
C5 = dict(experts=256, top_k=8, hidden=2048, inter=512, tokens=(1, 16, 256), zipf=1.1)
Q4_EXPERT_BYTES = lambda H, I: 3 * I * (H // 32) * 18                           # gate + up + down
FP4_EXPERT_BYTES = lambda H, I: 3 * (I * H // 2 + I * H // 32)                   # split weight + E8M0


def _graph_time(stream, phases, steps, warmup):
    """Captures one CUDA graph per phase (each phase enqueues one step on
    `stream`), replays `warmup` then `steps` steps round-robin; returns the
    device time of the timed steps (ms, CUDA events on `stream`)."""
    import torch
    graphs = []
    for fn in phases:
        with torch.cuda.stream(stream):
            fn()  # outside capture first: workspaces, kernel attributes
    torch.cuda.synchronize()
    for fn in phases:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        graphs.append(g)
    for i in range(warmup):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        with torch.cuda.stream(stream):
            graphs[(warmup + i) % len(graphs)].replay()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    del graphs
    return ms


def _q4_experts(qb, n, H, I, O, gen, dev):
    import torch
    from objeta_b200 import QGemvShape, QuantFormat
    mats = {"gate": [], "up": [], "down": []}
    for _ in range(n):
        for name, (r, c) in (("gate", (I, H)), ("up", (I, H)), ("down", (O, I))):
            m = torch.randn(r, c, device=dev, generator=gen) * 0.02
            mats[name].append(qb.quantize_matrix_device(QuantFormat.Q4_0, m, QGemvShape.new(QuantFormat.Q4_0, r, c)))
            del m
    return mats


def bench_c3(qb, dev, gen, steps, warmup, peak):
    """4 Q4_0 layers, 8 experts, top-2 (renormalised), H 4096,
    I 14336, one token; each layer's output is the next layer's input."""
    import torch
    from objeta_b200.moe import MoeLayer
    c = C3
    H, I, L, E, K = c["hidden"], c["inter"], c["layers"], c["experts"], c["top_k"]
    layers = []
    for _ in range(L):
        m = _q4_experts(qb, E, H, I, H, gen, dev)
        layers.append(MoeLayer(0, H, I, H, m["gate"], m["up"], m["down"]))
    S = 8
    logits = torch.randn(S, L, E, device=dev, generator=gen)
    x0 = torch.randn(S, H, device=dev, generator=gen)
    bufs = [torch.empty(H, device=dev) for _ in range(2)]
    ids = [torch.empty(K, dtype=torch.int32, device=dev) for _ in range(L)]
    ws = [torch.empty(K, device=dev) for _ in range(L)]
    stream = torch.cuda.Stream(device=dev)

    def phase(sidx):
        def fn():
            x = x0[sidx]
            for li, layer in enumerate(layers):
                layer.forward(logits[sidx, li], K, x, renormalize=True, d_out=bufs[li % 2], stream=stream,
                              ids=ids[li], weights=ws[li])
                x = bufs[li % 2]
        return fn
    ms = _graph_time(stream, [phase(i) for i in range(S)], steps, warmup)
    per_tok = ms / steps
    nbytes = L * K * Q4_EXPERT_BYTES(H, I)
    gbs = nbytes / (per_tok / 1e3) / 1e9
    del layers
    torch.cuda.empty_cache()
    return {"config": "configs[2] Q4_0 MoE stack: 4 layers x top-2 of 8, H 4096, I 14336, 1 token",
            "tokens_per_s": round(1e3 / per_tok, 1), "us_per_token": round(per_tok * 1e3, 2),
            "weight_bytes_per_token": nbytes, "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 4),
            # per layer: router, gate/up (x image built in-kernel), activation image, down
            "launches_per_token": L * 4, "l2_defeat": "198 MB of experts per layer, 8 routing phases",
            "steps": steps}


def run_moe_config(args, local):
    """One MoE config alone (configs[2], configs[3], or configs[4] with the
    expert cache, one rank), timed as in the full bench line."""
    import torch
    from objeta_b200 import QuantBackend
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(1234)
    peak, _ = read_peaks()
    steps = max(3, min(args.steps, 20))
    if args.moe_config == "c3":
        return {"c3_q4_stack": bench_c3(QuantBackend(local), dev, gen, steps, args.warmup, peak)}
    if args.moe_config == "c5cache":
        return {"c5_ep_cache": bench_c5_cache(QuantBackend(local), dev, gen, 1, 0, None, steps, args.warmup, peak)}
    return {"c4_fp4_shared": bench_c4(dev, gen, steps, args.warmup, peak)}


def bench_c4(dev, gen, steps, warmup, peak):
    """256 split-FP4 experts (codes uniform, E8M0 scales
    2^-8..2^-4), H 4096, I 2048, router top-8 (renormalised), plus one bf16
    shared expert added onto the routed output; one token."""
    import torch
    from objeta_b200.moe import MoeLayer, ffn_bf16_device
    c = C4
    H, I, E, K = c["hidden"], c["inter"], c["experts"], c["top_k"]
    t = {n: [] for n in ("gw", "gs", "uw", "us", "dw", "ds")}
    for _ in range(E):
        for wn, sn, r, cc in (("gw", "gs", I, H), ("uw", "us", I, H), ("dw", "ds", H, I)):
            t[wn].append(torch.randint(0, 256, (r * cc // 2,), device=dev, dtype=torch.uint8, generator=gen))
            t[sn].append(torch.randint(119, 124, (r * cc // 32,), device=dev, dtype=torch.uint8, generator=gen))
    layer = MoeLayer(3, H, I, H, t["gw"], t["uw"], t["dw"], t["gs"], t["us"], t["ds"])
    # the shared expert: bf16 ~ N(0, 0.02^2), added onto the routed output
    sh = [(torch.randn(r, cc, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
          for r, cc in ((I, H), (I, H), (H, I))]
    S = 8
    logits = torch.randn(S, E, device=dev, generator=gen)
    x0 = torch.randn(S, H, device=dev, generator=gen)
    out = torch.empty(H, device=dev)
    ids = torch.empty(K, dtype=torch.int32, device=dev)
    ws = torch.empty(K, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def phase(sidx):
        def fn():
            layer.forward(logits[sidx], K, x0[sidx], renormalize=True, d_out=out, stream=stream, ids=ids,
                          weights=ws)
            ffn_bf16_device(sh[0], sh[1], sh[2], H, I, H, x0[sidx], out, accumulate=True, stream=stream)
        return fn
    ms = _graph_time(stream, [phase(i) for i in range(S)], steps, warmup)
    per_tok = ms / steps
    nbytes = K * FP4_EXPERT_BYTES(H, I) + 3 * I * H * 2
    gbs = nbytes / (per_tok / 1e3) / 1e9
    del layer, t
    torch.cuda.empty_cache()
    return {"config": "configs[3]: 256 split FP4 E2M1 + E8M0 experts top-8 plus 1 bf16 shared expert, H 4096, "
                      "I 2048, 1 token (out = routed combine + shared)",
            "tokens_per_s": round(1e3 / per_tok, 1), "us_per_token": round(per_tok * 1e3, 2),
            "weight_bytes_per_token": nbytes, "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 4),
            # routed: router, x image, gate/up, activation image, down; shared: gate/up, down (x read directly)
            "launches_per_token": 7, "l2_defeat": "8 routing phases x 107 MB routed + 50 MB shared", "steps": steps}


def zipf_routes(T, E, K, s, perm, rng):
    """Top-k expert ids per token drawn from Zipf(s) over the permutation
    `perm` (rank i -> expert perm[i]), distinct within a token; weights are
    a softmax of N(0,1) over the k picks."""
    p = 1.0 / np.arange(1, E + 1) ** s
    p /= p.sum()
    ids = np.stack([perm[rng.choice(E, K, replace=False, p=p)] for _ in range(T)]).astype(np.int32)
    lg = rng.standard_normal((T, K))
    w = np.exp(lg - lg.max(1, keepdims=True))
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    return ids, w


def bench_c5_resident(qb, dev, gen, world, rank, group, steps, warmup, peak):
    """configs[4] expert-parallel layer, all of this rank's experts resident:
    256 Q4_0 experts block-partitioned over the ranks, H 2048, I 512, top-8
    Zipf(1.1) routing, T tokens per rank, NCCL all-to-all dispatch/combine."""
    import torch
    import torch.distributed as dist
    from objeta_b200.ep import ExpertParallelMoe, ep_packed_rows
    from objeta_b200.moe import MoeLayer
    c = C5
    H, I, E, K = c["hidden"], c["inter"], c["experts"], c["top_k"]
    epr = E // world
    # every rank builds the same experts from the same seed, keeps its block
    g = torch.Generator(device=dev).manual_seed(4242)
    m = _q4_experts(qb, E, H, I, H, g, dev)
    sl = slice(rank * epr, (rank + 1) * epr)
    layer = MoeLayer(0, H, I, H, m["gate"][sl], m["up"][sl], m["down"][sl])
    del m
    torch.cuda.empty_cache()
    perm = np.random.default_rng(7).permutation(E)
    ep = ExpertParallelMoe(layer, E, K, rank=rank, world=world, group=group)
    res = {}
    for T in c["tokens"]:
        rng = np.random.default_rng(1000 * T + rank)
        S = 4
        xs = [torch.randn(T, H, device=dev, generator=gen) for _ in range(S)]
        routes = [zipf_routes(T, E, K, c["zipf"], perm, rng) for _ in range(S)]
        ids = [torch.from_numpy(r[0]).to(dev) for r in routes]
        ws = [torch.from_numpy(r[1]).to(dev) for r in routes]
        n = max(3, min(steps, 10))
        # weight bytes each step must read: this rank's distinct experts
        # (host dispatch plans, outside the timing)
        plans = [ep.plan(ids[i]) for i in range(S)]
        uniq = sum(len(np.unique(plans[i % S].pair_expert)) for i in range(n))
        nvb = 0
        # the step has no host round trip (one rank: device sort; several: the
        # device exchange, its NCCL all-gathers and all-to-all on the step's
        # stream), so every rank captures it in CUDA graphs and replays them;
        # the graphs are released before the process group is destroyed
        stream = torch.cuda.Stream(device=dev)
        if world > 1:
            dist.barrier(group=group)
        ms = _graph_time(stream, [(lambda i=i: ep.forward(xs[i], ids[i], ws[i])) for i in range(S)], n, warmup)
        stats = torch.tensor([ms, uniq * Q4_EXPERT_BYTES(H, I), nvb], dtype=torch.float64, device=dev)
        if world > 1:
            mx = stats.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
            dist.all_reduce(stats, op=dist.ReduceOp.SUM, group=group)
            ms = float(mx[0])
        per_step = ms / n
        wbytes = float(stats[1]) / n
        gbs = wbytes / (per_step / 1e3) / 1e9
        phases = ep_phases(ep, xs, ids, ws, dev, group, world)
        # bytes each rank receives over NVLink per step: the packed buffers of
        # the G - 1 other ranks (one all-gather) and their partials (one
        # all-to-all); nothing at one rank
        rows = ep_packed_rows(T, K, H)
        nv_rank = (world - 1) * (rows * H + T * H) * 4
        coll_us = phases.get("pack+all_gather", 0.0) + phases.get("all_to_all", 0.0)
        res[f"T{T}"] = {"tokens_per_s": round(T * world * 1e3 / per_step, 1), "us_per_step": round(per_step * 1e3, 1),
                        "unique_expert_bytes_per_step_all_ranks": int(wbytes), "GB/s_all_ranks": round(gbs, 1),
                        "frac_of_aggregate_hbm": round(gbs / (peak * world), 4),
                        "nvlink_bytes_per_step_all_ranks": int(nv_rank * world),
                        "nvlink_GB/s_per_gpu_over_step": round(nv_rank / (per_step / 1e3) / 1e9, 2),
                        "nvlink_GB/s_per_gpu_in_collectives": round(nv_rank / (coll_us / 1e6) / 1e9, 2)
                        if coll_us > 0 and nv_rank else 0.0,
                        "nvlink_frac_of_peer_copy_in_collectives": round(nv_rank / (coll_us / 1e6) / 1e9 / NVLINK_GBS, 4)
                        if coll_us > 0 and nv_rank else 0.0,
                        "phases_us": phases, "steps": n}
    del ep, layer
    torch.cuda.empty_cache()
    return {"config": f"configs[4] EP layer, experts resident: 256 Q4_0 experts / {world} rank(s), H 2048, I 512, "
                      "top-8 Zipf(1.1), T tokens per rank",
            "scaling": "weak (T tokens per rank)", "timer": "CUDA events around whole steps, max over ranks; the "
            "device-only step replayed as CUDA graphs (one rank: sort + pairs + combine; several: one NCCL "
            "all-gather of the packed token rows, ids and weights, device-built pair list, pairs, partial "
            "combine, one NCCL all-to-all, ordered sum); phases_us from CUDA events at the phase boundaries "
            "of 3 eager steps", **res}


NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool (nominal 900)


def ep_phases(ep, xs, ids, ws, dev, group, world, reps=3):
    """Mean device time (us) of each phase of an expert-parallel step, from
    CUDA events the layer records at its phase boundaries during `reps`
    eager (not graph) steps; max over ranks."""
    import torch
    import torch.distributed as dist
    sums = {}
    for i in range(reps):
        ep.phase_events = []
        ep.forward(xs[i % len(xs)], ids[i % len(ids)], ws[i % len(ws)])
        torch.cuda.synchronize()
        evs = ep.phase_events
        for (_, a), (name, b) in zip(evs, evs[1:]):
            sums[name] = sums.get(name, 0.0) + a.elapsed_time(b) * 1e3 / reps
    ep.phase_events = None
    names = sorted(sums)
    t = torch.tensor([sums[k] for k in names], dtype=torch.float64, device=dev)
    if world > 1 and names:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return {k: round(float(v), 1) for k, v in zip(names, t.tolist())}


def ep_summary(c5, world):
    """The expert-parallel numbers lifted to the top of the bench line."""
    out = {"config": c5["config"], "ranks": world, "scaling": c5["scaling"]}
    for key in ("T1", "T16", "T256"):
        r = c5.get(key)
        if not r:
            continue
        ph = r.get("phases_us", {})
        out[key] = {k: r[k] for k in ("tokens_per_s", "us_per_step", "frac_of_aggregate_hbm",
                                       "nvlink_bytes_per_step_all_ranks", "nvlink_GB/s_per_gpu_over_step",
                                       "nvlink_GB/s_per_gpu_in_collectives",
                                       "nvlink_frac_of_peer_copy_in_collectives")}
        out[key]["phases_us"] = ph
        if ph:
            out[key]["largest_phase"] = max(ph, key=ph.get)
    return out


def bench_c5_cache(qb, dev, gen, world, rank, group, steps, warmup, peak):
    """configs[4] as specified: this rank's 256 / G Q4_0 experts live in
    pinned host memory and reach the GPU through a CudaExpertCache holding
    25% of them (LRU + admission); T tokens per rank, Zipf(1.1) routing,
    NCCL all-to-all dispatch / combine.  Misses are PCIe uploads."""
    import torch
    import torch.distributed as dist
    from objeta_b200._lib import call
    from objeta_b200.ep import CachedExpertCompute, ExpertParallelMoe
    from objeta_b200.moe import CudaExpertCache, ExpertWeights, MoeExecutor
    c = C5
    H, I, E, K = c["hidden"], c["inter"], c["experts"], c["top_k"]
    epr = E // world
    g = torch.Generator(device=dev).manual_seed(4242)
    m = _q4_experts(qb, E, H, I, H, g, dev)
    sl = range(rank * epr, (rank + 1) * epr)
    host = []
    for e in sl:
        ts = [m[n][e].cpu().numpy() for n in ("gate", "up", "down")]
        for t in ts:
            call("objb_host_register", t.ctypes.data, t.nbytes)
        host.append(ExpertWeights(*ts))
    del m
    torch.cuda.empty_cache()
    # this box's pinned host -> device rate at the cache's copy size (one
    # expert tensor), the same copies the cache issues, back to back
    tens = [t for e in host for t in (e.w_gate, e.w_up, e.w_down)][:96]
    dbuf = torch.empty(max(t.nbytes for t in tens), dtype=torch.uint8, device=dev)
    srcs = [torch.from_numpy(t) for t in tens]
    h0 = torch.cuda.Event(enable_timing=True)
    h1 = torch.cuda.Event(enable_timing=True)
    for rep in range(2):
        h0.record()
        for t in srcs:
            dbuf[:t.numel()].copy_(t, non_blocking=True)
        h1.record()
        torch.cuda.synchronize()
    h2d_gbs = sum(t.numel() for t in srcs) / (h0.elapsed_time(h1) / 1e3) / 1e9
    del dbuf, srcs
    ebytes = Q4_EXPERT_BYTES(H, I)
    cap_experts = max(1, epr // 4)
    cache = CudaExpertCache(cap_experts * ebytes, rank if world > 1 else torch.cuda.current_device())
    ex = MoeExecutor(torch.cuda.current_device())
    comp = CachedExpertCompute(ex, cache, host, H, I, H)
    ep = ExpertParallelMoe(None, E, K, rank=rank, world=world, group=group, out_dim=H, compute=comp)
    perm = np.random.default_rng(7).permutation(E)
    res = {}
    for T in c["tokens"]:
        rng = np.random.default_rng(2000 * T + rank)
        S = 4
        xs = [torch.randn(T, H, device=dev, generator=gen) for _ in range(S)]
        routes = [zipf_routes(T, E, K, c["zipf"], perm, rng) for _ in range(S)]
        ids = [torch.from_numpy(r[0]).to(dev) for r in routes]
        ws = [torch.from_numpy(r[1]).to(dev) for r in routes]
        n = max(3, min(steps, 10))
        for i in range(warmup):
            ep.forward(xs[i % S], ids[i % S], ws[i % S])
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(group=group)
        st0 = cache.stats()
        loaded = reused = 0
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(n):
            ep.forward(xs[i % S], ids[i % S], ws[i % S])
            tel = comp.last_telemetry
            if tel is not None:
                loaded += tel.actual_expert_bytes_loaded
                reused += tel.resident_cache_bytes_reused
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1)
        st1 = cache.stats()
        stats = torch.tensor([ms, loaded, reused], dtype=torch.float64, device=dev)
        if world > 1:
            mx = stats.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
            dist.all_reduce(stats, op=dist.ReduceOp.SUM, group=group)
            ms = float(mx[0])
        per_step = ms / n
        hits = st1["hit_count"] - st0["hit_count"]
        misses = st1["miss_count"] - st0["miss_count"]
        res[f"T{T}"] = {"tokens_per_s": round(T * world * 1e3 / per_step, 1), "us_per_step": round(per_step * 1e3, 1),
                        "pcie_bytes_per_step_all_ranks": int(float(stats[1]) / n),
                        "cache_reused_bytes_per_step_all_ranks": int(float(stats[2]) / n),
                        "pcie_GB/s_all_ranks": round(float(stats[1]) / n / (per_step / 1e3) / 1e9, 1),
                        "pcie_frac_of_measured_h2d": round(float(stats[1]) / n / (per_step / 1e3) / 1e9 / world
                                                           / h2d_gbs, 3),
                        "rank0_tensor_hit_rate": round(hits / max(1, hits + misses), 3), "steps": n}
    for e in host:
        for t in (e.w_gate, e.w_up, e.w_down):
            call("objb_host_unregister", t.ctypes.data)
    del ep, comp, cache, ex
    torch.cuda.empty_cache()
    return {"config": f"configs[4] EP layer with expert cache: 256 Q4_0 experts / {world} rank(s) in pinned host "
                      f"memory, cache = {cap_experts} experts per GPU (25%), H 2048, I 512, top-8 Zipf(1.1), "
                      "T tokens per rank",
            "bound": "PCIe (cache misses) + HBM", "scaling": "weak (T tokens per rank)",
            "h2d_pinned_GB/s_per_gpu": round(h2d_gbs, 1),
            "h2d_note": "measured on each rank alone: 96 back-to-back copies of one expert tensor (576 KB) from "
                        "registered host memory; the fraction divides the per-GPU upload rate by it", **res}


# --------------------------------------------------------- reference arm
def run_reference(args, world, rank):
    """The reference's CPU path on the host cores: the oracle's C restatement
    of gemv_cpu over the configs[1] sweep, all host threads, `steps` passes
    after `warmup` (rank 0 only; other ranks exit without work)."""
    if rank != 0:
        return None
    legs = cpu_legs(args.steps, args.warmup)
    value = legs["value"]
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(legs["seconds_per_pass"] * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic, seeded",
            "config": sweep_config(world),
            "cpu_baseline": legs,
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_case(args, local):
    """One sweep case alone: W + K launches of GEMV `fmt:RxC` (weights rotated
    over >= 4x L2 copies), timed with CUDA events on the launching stream."""
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    from objeta_b200.quant import gemv_device
    name, _, dims = args.case.partition(":")
    fmt = {v: k for k, v in FMT_NAMES.items()}[name]
    rows, cols = (int(v) for v in dims.split("x"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    qb = QuantBackend(local)
    gen = torch.Generator(device=dev).manual_seed(1234)
    shape = QGemvShape.new(QuantFormat(fmt), rows, cols)
    m = torch.randn(rows, cols, device=dev, generator=gen) * 0.02
    q0 = qb.quantize_matrix_device(QuantFormat(fmt), m, shape)
    del m
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    copies = [q0] + [q0.clone() for _ in range(max(2, math.ceil(4 * l2 / q0.numel())) - 1)]
    x = torch.randn(cols, device=dev, generator=gen)
    y = torch.empty(rows, device=dev)
    stream = torch.cuda.Stream(device=dev)
    for i in range(args.warmup):
        gemv_device(fmt, copies[i % len(copies)], x, y, rows, cols, stream)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        gemv_device(fmt, copies[(args.warmup + i) % len(copies)], x, y, rows, cols, stream)
    t1.record(stream)
    torch.cuda.synchronize()
    us = t0.elapsed_time(t1) * 1e3 / args.steps
    return {"case": args.case, "launches": args.steps, "us_per_gemv": round(us, 2),
            "GB/s": round(algo_bytes(fmt, rows, cols) / us / 1e3, 1), "copies": len(copies)}


def run_grouped(args, local):
    """configs[4] pairs for T tokens: the grouped tensor-core path
    (moe_pairs_tc) and the CUDA-core pair programs (moe_pairs), W + K calls
    each on one stream, timed with CUDA events."""
    import torch
    from objeta_b200 import QuantBackend
    from objeta_b200.ep import moe_pairs, moe_pairs_tc
    from objeta_b200.moe import MoeLayer
    T = int(args.grouped)
    c = C5
    H, I, E, K = c["hidden"], c["inter"], c["experts"], c["top_k"]
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    qb = QuantBackend(local)
    gen = torch.Generator(device=dev).manual_seed(4242)
    m = _q4_experts(qb, E, H, I, H, gen, dev)
    layer = MoeLayer(0, H, I, H, m["gate"], m["up"], m["down"])
    rng = np.random.default_rng(1000 * T)
    ids, _ = zipf_routes(T, E, K, c["zipf"], np.random.default_rng(7).permutation(E), rng)
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable")
    pe = torch.from_numpy(flat[order].astype(np.int32)).to(dev)
    pt = torch.from_numpy((order // K).astype(np.int32)).to(dev)
    po = torch.from_numpy(order.astype(np.int32)).to(dev)
    x = torch.randn(T, H, device=dev, generator=gen)
    v = torch.empty(T * K, H, device=dev)
    stream = torch.cuda.Stream(device=dev)
    res = {"grouped_tokens": T, "pairs": T * K, "distinct_experts": int(len(np.unique(flat))),
           "unique_expert_bytes": int(len(np.unique(flat)) * Q4_EXPERT_BYTES(H, I))}
    for name, fn in (("tc", moe_pairs_tc), ("cuda_core", moe_pairs)):
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                fn(layer, pe, pt, x, v, pair_out=po, stream=stream)
            torch.cuda.synchronize()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(args.steps):
                fn(layer, pe, pt, x, v, pair_out=po, stream=stream)
            t1.record(stream)
        torch.cuda.synchronize()
        res[f"us_{name}"] = round(t0.elapsed_time(t1) * 1e3 / args.steps, 1)
    return res


def run_official(args, local):
    """Official routed experts for T tokens: grouped block-scaled pairs vs the
    per-token CUDA-core launch (objb_moe_official_selected_device)."""
    import torch
    from objeta_b200.ep import moe_combine, moe_pairs_official_tc
    from objeta_b200.moe import MoeLayer
    c = C4
    H, I, K = c["hidden"], c["inter"], c["top_k"]
    E = int(args.experts or c["experts"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(77)
    t = {n: [] for n in ("gw", "gs", "uw", "us", "dw", "ds")}
    for _ in range(E):
        for wn, sn, r, cc in (("gw", "gs", I, H), ("uw", "us", I, H), ("dw", "ds", H, I)):
            t[wn].append(torch.randint(0, 256, (r * cc // 2,), device=dev, dtype=torch.uint8, generator=gen))
            t[sn].append(torch.randint(119, 124, (r * cc // 32,), device=dev, dtype=torch.uint8, generator=gen))
    layer = MoeLayer(3, H, I, H, t["gw"], t["uw"], t["dw"], t["gs"], t["us"], t["ds"])
    ebytes = 3 * (I * H // 2 + I * H // 32)
    res = {"config": f"official routed experts: {E} split FP4 experts, H {H}, I {I}, top-{K}, Zipf(1.1) over a "
                     "seeded permutation, act_quant FP8 activations", "expert_bytes": ebytes}
    stream = torch.cuda.Stream(device=dev)
    for T in (int(v) for v in str(args.official).split(",")):
        rng = np.random.default_rng(3000 + T)
        ids, w = zipf_routes(T, E, K, 1.1, np.random.default_rng(7).permutation(E), rng)
        flat = ids.reshape(-1)
        order = np.argsort(flat, kind="stable")
        pe = torch.from_numpy(flat[order].astype(np.int32)).to(dev)
        pt = torch.from_numpy((order // K).astype(np.int32)).to(dev)
        po = torch.from_numpy(order.astype(np.int32)).to(dev)
        x = torch.randn(T, H, device=dev, generator=gen)
        dw = torch.from_numpy(w).to(dev)
        di = torch.from_numpy(ids.astype(np.int32)).to(dev)
        v = torch.empty(T * K, H, device=dev)
        out = torch.empty(T, H, device=dev)
        slot = torch.arange(T * K, dtype=torch.int32, device=dev).reshape(T, K)

        def grouped():
            moe_pairs_official_tc(layer, pe, pt, x, v, pair_out=po, stream=stream)
            moe_combine(v, slot, dw, out, stream=stream)

        def per_token():
            for i in range(T):
                layer.forward_official_selected(di[i], dw[i], x[i], d_out=out[i], stream=stream)

        row = {"distinct_experts": int(len(np.unique(flat))), "unique_expert_bytes": int(len(np.unique(flat)) * ebytes)}
        for name, fn in (("tc_grouped", grouped), ("cuda_core_per_token", per_token)):
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    fn()
                torch.cuda.synchronize()
                t0 = torch.cuda.Event(enable_timing=True)
                t1 = torch.cuda.Event(enable_timing=True)
                t0.record(stream)
                for _ in range(args.steps):
                    fn()
                t1.record(stream)
            torch.cuda.synchronize()
            us = t0.elapsed_time(t1) * 1e3 / args.steps
            row[f"us_{name}"] = round(us, 1)
            row[f"tokens_per_s_{name}"] = round(T * 1e6 / us, 1)
        res[f"T{T}"] = row
    return res


def main():
    # NCCL's own log lines (e.g. its version banner when NCCL_DEBUG is set)
    # go to stderr, so stdout carries only the result line.
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--case", default=None, help="fmt:RxC, e.g. q4_0:151936x2048 (one GEMV alone)")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE configs reported beside the headline")
    ap.add_argument("--official", default=None,
                    help="T[,T..]: official routed experts, grouped block-scaled pairs vs the per-token launch")
    ap.add_argument("--experts", type=int, default=None, help="expert count for --official (default configs[3])")
    ap.add_argument("--grouped", type=int, default=None,
                    help="T: the configs[4] pairs of T tokens on the grouped tensor-core path and the CUDA-core path")
    ap.add_argument("--moe-config", default=None, choices=["c3", "c4", "c5cache"],
                    help="run one MoE config alone (a few GB on the device: small enough for an ncu capture)")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (minimum)")
        args.warmup = 3
    world, rank, local = dist_env()
    if args.case:
        print(json.dumps(run_case(args, local)), flush=True)
        return
    if args.grouped:
        print(json.dumps(run_grouped(args, local)), flush=True)
        return
    if args.official:
        print(json.dumps(run_official(args, local)), flush=True)
        return
    if args.moe_config:
        print(json.dumps(run_moe_config(args, local)), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, world, rank)
    else:
        res = run_ours(args, world, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
