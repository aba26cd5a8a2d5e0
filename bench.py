"""Benchmark: KTIR kernel executions per second on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl reference]
                    [--replicas] [--only]

A step is one execution of a KTIR function (one pass of the hot path over one
input set).  The headline workload is the largest single-GPU configuration,
causal multi-head attention B4 H32 S2048 D128 on a 32-core grid (--config
picks another).  The same line carries `per_config`: the same measurements
for all five benchmark workloads (attention, gemm, softmax, gather_add,
vector_add), unless --only.

value   executions/s with inputs resident in HBM, whole job (all ranks), timed
        with CUDA events over K steps; steps rotate over buffer sets whose
        total exceeds the 126 MB L2, so every step reads from HBM.
long_window  the same steps repeated for at least 10 ms of device time.
e2e     executions/s through KTIRInterpreter.execute_function with host NumPy
        arrays: upload of every tensor argument, run, download of the results
        inside the timed region.
roofline  the dominant kernel's algorithmic bytes (or flops) per execution
        over its measured time per execution, against MEASURED_PEAKS.json.
cpu_baseline  the NumPy oracle (a restatement of the reference interpreter)
        timed on this host on a bounded sample of the same workload (N=1).

Multi-GPU: one process per GPU (torchrun); by default one execution's core
grid is split across the ranks by contiguous core ranges (strong scaling);
the attention split passes K/V blocks between the GPUs in a ring over NVLink.
--replicas runs one whole execution per rank instead (weak scaling).  Times
are the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from ktir_cpu_b200 import workloads as W  # noqa: E402

METRIC = "ktir_execs_per_sec"
UNIT = "execs/s"
HEADLINE = "attention"
ORDER = ["attention", "gemm", "softmax", "gather_add", "vector_add"]
L2_BYTES = 126 * 1024 * 1024
QUEUE_CYCLES = 4_000_000      # device spin ahead of each timed window

# algorithmic work per execution (bytes for HBM-bound, flops for tensor-bound)
WORK = {
    "vector_add": ("hbm", 3 * 1024 * 2),
    "softmax": ("hbm", 2 * 4096 * 1024 * 2),
    "gather_add": ("hbm", 262144 * 4 + 2 * 262144 * 128 * 2),
    "gemm": ("tensor", 2 * 4096 ** 3),
    "attention": ("tensor", 4 * 4 * 32 * 2048 * 2048 * 128 // 2),
}
DOMINANT = {"vector_add": "k_ew_bin_f16", "softmax": "k_softmax_rows", "gather_add": "k_rmw_apply",
            "gemm": "k_gemm_tcgen05", "attention": "k_fmha_tcgen05"}
WORKLOAD = {"softmax": "row softmax f16 [4096,1024], grid 32, 128 rows/core, f32 max/sum",
            "vector_add": "add_kernel f16 (1024,)",
            "gemm": "GEMM f16 4096^3, f32 accumulate, grid 8x4, 512x1024 per core",
            "gather_add": "indirect gather/+1.0/RMW-scatter, table f16 [1048576,128], "
                          "262144 i32 indices, grid 64",
            "attention": "causal MHA B4 H32 S2048 D128 f16, grid 32: 4 head groups, each "
                         "a ring of 8 cores that own zigzag query-block pairs"}


def peaks():
    """(HBM GB/s, burst TFLOP/s, sustained TFLOP/s, source).  The timed region
    follows 1.5 s of the same launches, so a tensor-core kernel is timed in the
    power-capped steady state: its roofline uses the sustained GEMM figure (the
    burst fraction is reported beside it)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return (d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


# variants measured beside the five workloads when the grid is split over GPUs:
# the attention program with cores that own whole heads (no K/V exchange)
VARIANTS = {"attention_heads": ("attention", {"layout": "heads", "groups": 1})}
WORKLOAD["attention_heads"] = ("causal MHA B4 H32 S2048 D128 f16, grid 32, cores own whole "
                               "heads")


def base_of(name: str):
    """(workload, extra KTIR generator parameters) of a bench entry."""
    return VARIANTS.get(name, (name, {}))


def config_dict(name: str, world: int, mode: str):
    """The workload's description; both arms emit exactly this dict."""
    if world == 1:
        par = "single GPU"
    elif mode == "replicas":
        par = f"replicas x{world}"
    else:
        par = f"core grid split over {world} GPUs by contiguous core ranges"
    base, extra = base_of(name)
    params = dict(W.FULL[base], **extra)
    return {"workload": WORKLOAD[name], "name": name,
            "params": {k: (list(v) if isinstance(v, tuple) else v) for k, v in params.items()},
            "parallelism": par}


class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for n, v in zip(names, s[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.samples)}


def cpu_baseline(config: str, budget_s: float = 10.0):
    """Time the NumPy oracle on a bounded sample of one execution and scale it
    to a whole execution: the leading cores, or a leading share of the first
    core's outermost loop when one core alone exceeds the budget (cores and
    loop iterations are uniform in these workloads)."""
    from oracle.interp import OracleInterpreter
    src = W.source(config)
    kw = W.inputs(config, seed=0)
    fname = W.FUNC[config]

    def run(cores, loops):
        o = OracleInterpreter()
        o.load(src)
        o.core_limit, o.loop_limit = cores, loops
        t0 = time.perf_counter()
        o.execute_function(fname, **{k: v.copy() for k, v in kw.items()})
        return time.perf_counter() - t0, o
    # probe: the first iteration of the first core
    t_probe, o = run(1, 1)
    n_cores = o.n_cores
    frac_probe = o.loop_fraction
    per_core = t_probe / frac_probe
    if per_core <= budget_s:
        k = int(max(1, min(n_cores, budget_s / max(per_core, 1e-6))))
        t, o = run(k, None)
        per_exec = t * n_cores / k
        sample = (f"{k} of {n_cores} cores of one {config} execution, scaled linearly"
                  if k < n_cores else f"one full {config} execution")
    else:
        iters = max(1, int(budget_s / max(t_probe, 1e-6)))
        t, o = run(1, iters)
        per_exec = t / o.loop_fraction * n_cores
        sample = (f"{o.loop_fraction:.3g} of the outermost loop of core 0 of {n_cores} cores "
                  f"of one {config} execution, scaled linearly")
    return {"value": 1.0 / per_exec, "unit": UNIT, "cores": 1, "kind": "port", "sample": sample,
            "seconds_per_exec": per_exec}


def run_reference(args, world):
    """The reference arm: the NumPy oracle port of the reference interpreter
    on this host's cores, one bounded sample per step (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    t_start = time.perf_counter()
    mode = "replicas" if args.replicas else "split"
    names = [args.config] + ([] if args.only else [n for n in ORDER if n != args.config])
    per = {}
    for name in names:
        n_steps = args.warmup + args.steps if name == args.config else 2
        budget = max(0.2, 60.0 / (args.warmup + args.steps)) if name == args.config else 5.0
        vals = []
        for i in range(n_steps):
            cb = cpu_baseline(name, budget_s=budget)
            if name != args.config or i >= args.warmup:
                vals.append(cb["value"])
        v = float(np.mean(vals))
        per[name] = {"value": v, "unit": UNIT, "ms_per_step": 1000.0 / v,
                     "config": config_dict(name, world, mode),
                     "cpu_baseline": {"value": v, "unit": UNIT, "cores": 1, "kind": "port",
                                      "sample": cb["sample"]}}
    h = per[args.config]
    line = {"metric": METRIC, "value": h["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": h["ms_per_step"],
            "higher_is_better": True, "scaling": "weak" if mode == "replicas" else "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": h["config"], "impl": "reference", "cpu_baseline": h["cpu_baseline"],
            "e2e": {"value": h["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t_start}
    if not args.only:
        line["per_config"] = per
    print(json.dumps(line), flush=True)


def read_traffic(config):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", f"{DOMINANT[config]}_{config}.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1])
                except ValueError:
                    return None
    return None


class Env:
    """Process-wide state of one bench run (rank, device, process group)."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.mode = "replicas" if (args.replicas or self.world == 1) else "split"
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, *vals):
        if self.world == 1:
            return [float(v) for v in vals]
        t = self.torch.tensor([float(v) for v in vals], device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(x) for x in t.tolist()]


def _busy(exe, sets, stream, seconds, dev, torch):
    """Keep the GPU on this workload for `seconds` (clock sampling, power-cap
    steady state before a tensor-core kernel is timed).  A plan that exchanges
    data between ranks runs a fixed number of executions instead, so every
    rank issues the same collectives."""
    if exe.plan.collective:
        for i in range(int(seconds * 200)):
            exe.launch(sets[i % len(sets)][0], stream, sets[i % len(sets)][1])
        torch.cuda.synchronize(dev)
        return
    t_end = time.time() + seconds
    i = 0
    while time.time() < t_end:
        for _ in range(20):
            exe.launch(sets[i % len(sets)][0], stream, sets[i % len(sets)][1])
            i += 1
        torch.cuda.synchronize(dev)


def measure_batched(env: Env, exe, host, steps: int, n: int = 65536):
    """B independent add_kernel executions per launch (Executable.batched):
    the GB/s figure of the 6 KB workload.  n * 6 KB = 384 MiB per launch, three
    times the L2."""
    torch = env.torch
    bx = exe.batched(n)
    ts = []
    for arr in host:
        t = torch.empty(arr.nbytes * n, dtype=torch.uint8, device=env.dev)
        t.view(n, arr.nbytes).copy_(torch.from_numpy(arr.view(np.uint8).reshape(1, -1)).expand(n, -1))
        ts.append(t)
    bufs = bx.buffers(ts)
    stream = torch.cuda.current_stream(env.dev)
    for _ in range(3):
        bx.launch(ts, stream, bufs)
    torch.cuda.synchronize(env.dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        bx.launch(ts, stream, bufs)
    b.record(stream)
    torch.cuda.synchronize(env.dev)
    ms = a.elapsed_time(b) / steps
    (ms,) = env.max_over_ranks(ms)
    hbm_peak = peaks()[0]
    gbs = n * WORK["vector_add"][1] / (ms / 1000.0) / 1e9
    per_rank = 1 if (env.mode == "split" and env.world > 1) else env.world
    return {"executions_per_launch": n, "value": per_rank * n / (ms / 1000.0), "unit": UNIT,
            "ms_per_launch": ms, "gpu_launches": steps * len(bx.progs),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": gbs / hbm_peak, "kernel": "k_ew_bin_f16",
                         "traffic": read_traffic("vector_add")}}


def measure(env: Env, name: str, steps: int, with_cpu: bool):
    """Device-resident and end-to-end executions/s of one workload."""
    torch = env.torch
    from ktir_cpu_b200 import KTIRInterpreter
    args, dev, world, rank = env.args, env.dev, env.world, env.rank
    split = env.mode == "split" and world > 1
    base, extra = base_of(name)
    src = W.source(base, **extra)
    fname = W.FUNC[base]
    kw = W.inputs(base, seed=0 if split else rank)
    interp = KTIRInterpreter(device=dev, shard=(rank, world, None) if split else None)
    interp.load(src)
    # first call traces + lowers (cached) and runs the path once
    interp.execute_function(fname, **{k: v.copy() for k, v in kw.items()})
    exe = interp.last_executable
    plan = exe.plan

    # --- device-resident timed region ------------------------------------------
    host = [interp.memory.hbm.allocs[a] for a in sorted(interp.memory.hbm.allocs)]
    set_bytes = sum(int(a.nbytes) for a in host)
    n_sets = max(2, int(math.ceil(2 * L2_BYTES / max(set_bytes, 1))))
    n_sets = min(n_sets, 64) if not args.profile else 2
    sets = []
    for _ in range(n_sets):
        ts = []
        for arr in host:
            t = torch.empty(arr.nbytes + 16, dtype=torch.uint8, device=dev)
            t[:arr.nbytes].copy_(torch.from_numpy(arr.view(np.uint8).reshape(-1)))
            ts.append(t)
        sets.append((ts, exe.buffers(ts)))
    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
    torch.cuda.synchronize(dev)
    if args.profile:
        for i in range(steps):
            exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
        torch.cuda.synchronize(dev)
        out = {"profile_run": name, "plan": plan.kind,
               "launches": (args.warmup + steps) * plan.kernel_launches}
        if name == "vector_add" and not split:
            # then the batched variant: warmup + steps launches of 65536 executions
            b = measure_batched(env, exe, host, steps)
            out["batched_launches"] = 3 + steps + b["gpu_launches"]
        return out
    # a workload too small for its rotating sets to exceed L2 is timed with an
    # L2 flush (a 256 MiB write) before every execution instead, each
    # execution between its own pair of events
    flush = n_sets * set_bytes < 2 * L2_BYTES
    # the K timed executions, recorded once as a CUDA graph so the host's
    # per-launch cost does not pace the device (plans with an NCCL exchange
    # keep plain launches)
    graph = None
    if not plan.collective and not args.eager and not flush:
        graph = exe.capture([sets[i % n_sets][0] for i in range(steps)])
        graph.replay()
        torch.cuda.synchronize(dev)

    def run_steps():
        if graph is not None:
            graph.replay()
        else:
            for i in range(steps):
                exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])

    if flush:
        scrub = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)

        def flushed(n):
            """Device ms of n executions, each after an L2 flush."""
            evs = []
            for i in range(n):
                scrub.fill_(i & 255)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
                b.record(stream)
                evs.append((a, b))
            torch.cuda.synchronize(dev)
            return float(sum(a.elapsed_time(b) for a, b in evs))

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    env.barrier()
    with ClockSampler(env.local) as clk:
        # keep the GPU busy until the sampler is producing samples, so the
        # clocks recorded are the clocks under this load
        _busy(exe, sets, stream, 1.5, dev, torch)
        env.barrier()
        torch.cuda.synchronize(dev)
        # a device-side wait (about 2 ms) ahead of the start event, so the
        # host has queued the K steps (or submitted the whole graph of them)
        # before the clock starts: the host's launch latency is not device time
        torch.cuda._sleep(QUEUE_CYCLES)
        if flush:
            k_ms = flushed(steps)
        else:
            ev[0].record(stream)
            run_steps()
            ev[1].record(stream)
            torch.cuda.synchronize(dev)
            k_ms = ev[0].elapsed_time(ev[1])
        # a second window of at least 10 ms of device time: the K steps repeated
        reps = max(1, int(math.ceil(10.0 / max(k_ms, 1e-3))))
        env.barrier()
        torch.cuda._sleep(QUEUE_CYCLES)
        if flush:
            long_ms = flushed(steps * reps)
        else:
            ev[2].record(stream)
            for _ in range(reps):
                run_steps()
            ev[3].record(stream)
            torch.cuda.synchronize(dev)
            long_ms = ev[2].elapsed_time(ev[3])
        # per-execution event pairs, each execution alone between its events
        pairs = []
        for i in range(min(steps, 50)):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
            b.record(stream)
            pairs.append((a, b))
        torch.cuda.synchronize(dev)
        _busy(exe, sets, stream, 0.3, dev, torch)
    iso_ms = float(np.mean([a.elapsed_time(b) for a, b in pairs]))
    k_ms, long_ms, iso_ms = env.max_over_ranks(k_ms, long_ms, iso_ms)
    per_step_execs = 1 if split else world
    value = per_step_execs * steps / (k_ms / 1000.0)
    long_value = per_step_execs * steps * reps / (long_ms / 1000.0)

    # --- end to end through the public API ------------------------------------
    e2e_steps = args.e2e_steps or max(3, min(steps, 20))
    for _ in range(max(1, args.warmup)):
        interp.execute_function(fname, **kw)
    torch.cuda.synchronize(dev)
    env.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        interp.execute_function(fname, **kw)
    torch.cuda.synchronize(dev)
    e2e_s = time.perf_counter() - t0
    e2e_exe = interp.last_executable
    (e2e_s,) = env.max_over_ranks(e2e_s)
    e2e = per_step_execs * e2e_steps / e2e_s

    hbm_peak, tc_peak, tc_sustained, src_peak = peaks()
    bound, work = WORK[base]
    if split:
        work = work / world   # each rank's share of one execution
    kern_ms = k_ms / steps
    if bound == "hbm":
        achieved = work / (kern_ms / 1000.0) / 1e9
        peak, unit = hbm_peak, "GB/s"
    else:
        achieved = work / (kern_ms / 1000.0) / 1e12
        peak, unit = tc_sustained, "TFLOP/s"
    out = {
        "value": value, "unit": UNIT, "ms_per_step": k_ms / steps, "steps": steps,
        "config": config_dict(name, world, env.mode),
        "long_window": {"steps": steps * reps, "ms": long_ms, "value": long_value,
                        "ms_per_step": long_ms / (steps * reps)},
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak,
                     # the vector add's ncu capture is of a batched launch: its
                     # traffic belongs to the batched figure
                     "traffic": read_traffic(base) if base != "vector_add" else None,
                     "peak_source": src_peak + (" (sustained; timed after 1.5 s of load)"
                                                if bound == "tensor" else ""),
                     "frac_of_burst": (achieved / tc_peak if bound == "tensor" else None),
                     "kernel": DOMINANT[base], "kernel_ms": kern_ms,
                     "isolated_launch_ms": iso_ms, "plan_kernels": plan.kernel_launches},
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": e2e_exe.last_h2d_bytes,
                "d2h_bytes_per_step": e2e_exe.last_d2h_bytes,
                "arg_bytes": sum(v.nbytes for v in kw.values())},
        "gpu_launches": steps * plan.kernel_launches,
        "method": {"plan": plan.kind,
                   "l2": (f"flushed: a {2 * L2_BYTES >> 20} MiB write before every execution, "
                          f"each execution timed between its own events ({set_bytes} bytes "
                          f"of arguments, {n_sets} rotating sets)") if flush else
                         (f"{n_sets} rotating buffer sets of {set_bytes / 2**20:.1f} MiB "
                          f"(> 126 MB L2)"),
                   "launch": "cuda graph of the K steps" if graph is not None
                   else "host launch per step"},
        "clocks": clk.summary(),
    }
    if name == "vector_add" and not split:
        out["batched"] = measure_batched(env, exe, host, steps)
    if with_cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(base)
    # graphs are released before any process-group teardown
    del graph
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=HEADLINE, choices=sorted(W.FULL))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--only", action="store_true", help="measure the --config workload alone")
    ap.add_argument("--replicas", action="store_true",
                    help="N>1: one whole execution per rank (weak scaling) instead of a split")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--eager", action="store_true",
                    help="time per-step host launches instead of one CUDA graph of the K steps")
    ap.add_argument("--profile", action="store_true",
                    help="only warmup + steps plain launches on two buffer sets (for ncu)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        return run_reference(args, world)
    env = Env(args)
    if args.profile:
        r = measure(env, args.config, args.steps, with_cpu=False)
        if env.rank == 0:
            print(json.dumps(r), flush=True)
        return finish(env)
    head = measure(env, args.config, args.steps, with_cpu=True)
    per = {args.config: head}
    if not args.only:
        extra = list(VARIANTS) if env.mode == "split" and env.world > 1 else []
        for name in ORDER + extra:
            if name != args.config:
                per[name] = measure(env, name, args.steps, with_cpu=True)
    if env.rank == 0:
        line = {"metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": env.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
                "higher_is_better": True,
                "scaling": "strong" if env.mode == "split" and env.world > 1 else "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": head["config"], "roofline": head["roofline"], "e2e": head["e2e"],
                "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
                "long_window": head["long_window"], "method": head["method"]}
        if "cpu_baseline" in head:
            line["cpu_baseline"] = head["cpu_baseline"]
        if "batched" in head:
            line["batched"] = head["batched"]
        if not args.only:
            line["per_config"] = per
        print(json.dumps(line), flush=True)
    finish(env)


def finish(env):
    if env.world > 1:
        env.dist.barrier()
        env.dist.destroy_process_group()


if __name__ == "__main__":
    main()
