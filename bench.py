"""Benchmark: KTIR kernel executions per second on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl reference]

A step is one execution of a KTIR function (one pass of the hot path over one
input set).  Default workload: the 4096x1024 f16 row softmax on a 32-core
grid.  Other workloads (--config): vector_add, gemm, gather_add, attention.

value   executions/s with inputs resident in HBM, whole job (all ranks), timed
        with CUDA events; steps rotate over buffer sets whose total exceeds
        the 126 MB L2, so every step reads from HBM.
e2e     executions/s through KTIRInterpreter.execute_function with host NumPy
        arrays: upload of every tensor argument, run, download of every tensor
        argument inside the timed region.
roofline  the dominant kernel's algorithmic bytes (or flops) per launch over
        its average CUDA-event duration, against MEASURED_PEAKS.json.
cpu_baseline  the NumPy oracle (a restatement of the reference interpreter)
        timed on this host on a bounded sample of the same workload.

Multi-GPU: one process per GPU (torchrun); every rank executes its own full
call on its own inputs (replicas, weak scaling); time = max over ranks.
"""

from __future__ import annotations

import argparse
import json
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

# algorithmic work per execution (bytes for HBM-bound, flops for tensor-bound)
WORK = {
    "vector_add": ("hbm", 3 * 1024 * 2),
    "softmax": ("hbm", 2 * 4096 * 1024 * 2),
    "gather_add": ("hbm", 262144 * 4 + 2 * 262144 * 128 * 2),
    "gemm": ("tensor", 2 * 4096 ** 3),
    "attention": ("tensor", 4 * 4 * 32 * 2048 * 2048 * 128 // 2),
}
DOMINANT = {"vector_add": "k_ew", "softmax": "k_softmax_rows", "gather_add": "k_rmw_apply",
            "gemm": "k_gemm_tcgen05", "attention": "k_fmha_tcgen05"}


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


def cpu_baseline(config: str, budget_s: float = 20.0):
    """Time the NumPy oracle on a bounded sample (leading cores) and scale to one execution."""
    from oracle.interp import OracleInterpreter
    src = W.source(config)
    kw = W.inputs(config, seed=0)
    o = OracleInterpreter()
    o.load(src)
    fn = o.module.get_function(W.FUNC[config])
    n_cores = fn.num_cores
    # probe one core, then size the sample to the budget
    o.core_limit = 1
    t0 = time.perf_counter()
    o.execute_function(W.FUNC[config], **{k: v.copy() for k, v in kw.items()})
    t1 = time.perf_counter() - t0
    k = int(max(1, min(n_cores, budget_s / max(t1, 1e-6))))
    o.core_limit = k
    t0 = time.perf_counter()
    o.execute_function(W.FUNC[config], **{k2: v.copy() for k2, v in kw.items()})
    tk = time.perf_counter() - t0
    per_exec = tk * n_cores / k
    sample = (f"{k} of {n_cores} cores of one {config} execution, scaled linearly"
              if k < n_cores else f"one full {config} execution")
    return {"value": 1.0 / per_exec, "unit": UNIT, "cores": 1, "kind": "port", "sample": sample,
            "seconds_per_exec": per_exec}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = config_dict(args)
    t_start = time.perf_counter()
    vals = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(args.config, budget_s=max(2.0, 60.0 / max(1, args.warmup + args.steps)))
        if i >= args.warmup:
            vals.append(cb["value"])
    v = float(np.mean(vals))
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": cfg, "impl": "reference",
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": 1, "kind": "port",
                             "sample": cb["sample"]},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t_start}
    print(json.dumps(line), flush=True)


def config_dict(args):
    d = {"workload": {"softmax": "row softmax f16 [4096,1024], grid 32, 128 rows/core, f32 max/sum",
                      "vector_add": "add_kernel f16 (1024,)",
                      "gemm": "GEMM f16 4096^3, f32 accumulate, grid 8x4, 512x1024 per core",
                      "gather_add": "indirect gather/+1.0/RMW-scatter, table f16 [1048576,128], "
                                    "262144 i32 indices, grid 64",
                      "attention": "causal MHA B4 H32 S2048 D128 f16, grid 32"}[args.config],
         "name": args.config, "params": {k: (list(v) if isinstance(v, tuple) else v)
                                          for k, v in W.FULL[args.config].items()}}
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="softmax", choices=sorted(W.FULL))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--shard", action="store_true",
                    help="split one execution's core grid across the ranks (strong scaling)")
    ap.add_argument("--eager", action="store_true",
                    help="time per-step host launches instead of one CUDA graph of the K steps")
    ap.add_argument("--profile", action="store_true",
                    help="only warmup + steps plain launches on two buffer sets (for ncu)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist
    from ktir_cpu_b200 import KTIRInterpreter

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    src = W.source(args.config)
    fname = W.FUNC[args.config]
    kw = W.inputs(args.config, seed=0 if args.shard else rank)
    shard = (rank, world, None) if (args.shard and world > 1) else None
    interp = KTIRInterpreter(device=dev, shard=shard)
    interp.load(src)
    # first call traces + lowers (cached), and checks the path runs
    interp.execute_function(fname, **{k: v.copy() for k, v in kw.items()})
    exe = interp.last_executable
    plan = exe.plan

    # --- device-resident timed region -------------------------------------------
    nbytes = [int(b.nbytes) for b in exe.space.buffers]
    set_bytes = sum(nbytes)
    L2 = 126 * 1024 * 1024
    n_sets = max(2, int(np.ceil(2 * L2 / max(set_bytes, 1))))
    n_sets = min(n_sets, 64) if not args.profile else 2
    sets = []
    host = [interp.memory.hbm.allocs[a] for a in sorted(interp.memory.hbm.allocs)]
    for _ in range(n_sets):
        ts = []
        for arr in host:
            t = torch.empty(arr.nbytes + 16, dtype=torch.uint8, device=dev)
            t[:arr.nbytes].copy_(torch.from_numpy(arr.view(np.uint8)))
            ts.append(t)
        sets.append((ts, exe.buffers(ts)))
    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
    torch.cuda.synchronize(dev)
    if args.profile:
        for i in range(args.steps):
            exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
        torch.cuda.synchronize(dev)
        if rank == 0:
            print(json.dumps({"profile_run": args.config, "plan": plan.kind,
                              "launches": (args.warmup + args.steps) * plan.kernel_launches}))
        return
    # the K timed executions, recorded once as a CUDA graph so the host's
    # per-launch cost does not pace the device (plans with an NCCL exchange
    # keep plain launches)
    graph = None
    collective = any(l.kind == "allreduce_counts" for l in plan.launches)
    if not collective and not args.eager:
        graph = exe.capture([sets[i % n_sets][0] for i in range(args.steps)])
        graph.replay()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # keep the GPU busy until the sampler is producing samples, so the
        # clocks recorded are the clocks under this load
        t_end = time.time() + 1.5
        i = 0
        while time.time() < t_end:
            for _ in range(20):
                exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
                i += 1
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        # a short device-side wait ahead of the start event, so the host has
        # queued the K steps before the clock starts (the host's launch
        # latency is not device time)
        torch.cuda._sleep(200000)
        ev0.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        # per-launch durations of the plan's kernels (dominant kernel time)
        evs = []
        for i in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize(dev)
        t_end = time.time() + 0.3
        while time.time() < t_end:
            for _ in range(20):
                exe.launch(sets[i % n_sets][0], stream, sets[i % n_sets][1])
                i += 1
            torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    # average duration of the plan's kernels per step, from the events over
    # the timed region (one-kernel plans: the kernel itself); per-launch event
    # pairs are also reported but include the events' own overhead
    kern_ms = ms / args.steps
    launch_ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    if world > 1:
        t = torch.tensor([ms, kern_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kern_ms = float(t[0]), float(t[1])
    per_step_execs = 1 if shard else world
    value = per_step_execs * args.steps / (ms / 1000.0)

    # --- end to end through the public API ------------------------------------------
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 20))
    in_bytes = sum(v.nbytes for v in kw.values())
    # warm-up of the host path too (its page-locked result buffers are
    # allocated on first use and reused by later calls)
    for _ in range(max(1, args.warmup)):
        interp.execute_function(fname, **kw)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        interp.execute_function(fname, **kw)
    torch.cuda.synchronize(dev)
    e2e_s = time.perf_counter() - t0
    e2e_exe = interp.last_executable
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t[0])
    e2e = per_step_execs * e2e_steps / e2e_s

    if rank == 0:
        hbm_peak, tc_peak, tc_sustained, src_peak = peaks()
        bound, work = WORK[args.config]
        if shard:
            work = work / world   # each rank's share of one execution
        if bound == "hbm":
            achieved = work / (kern_ms / 1000.0) / 1e9
            peak, unit = hbm_peak, "GB/s"
        else:
            achieved = work / (kern_ms / 1000.0) / 1e12
            peak, unit = tc_sustained, "TFLOP/s"
        traffic = read_traffic(args.config)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if shard else "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": dict(config_dict(args), l2=f"{n_sets} rotating buffer sets of "
                           f"{set_bytes / 2**20:.1f} MiB (> 126 MB L2)", plan=plan.kind,
                           parallelism=(f"core grid split over {world} GPUs" if shard
                                        else f"replicas x{world}")),
            "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": src_peak + (" (sustained; timed after 1.5 s of load)"
                                                    if bound == "tensor" else ""),
                         "frac_of_burst": (achieved / tc_peak if bound == "tensor" else None),
                         "kernel": DOMINANT[args.config],
                         "kernel_ms": kern_ms, "isolated_launch_ms": launch_ms,
                         "plan_kernels": plan.kernel_launches,
                         "launch": "cuda graph of the K steps" if graph is not None
                         else "host launch per step"},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": e2e_exe.last_h2d_bytes,
                    "d2h_bytes_per_step": e2e_exe.last_d2h_bytes,
                    "arg_bytes": in_bytes},
            "gpu_launches": args.steps * plan.kernel_launches,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.config)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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


if __name__ == "__main__":
    main()
