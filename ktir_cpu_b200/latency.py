"""Analytic latency report for a KTIR call, computed on the host from the trace.

The reference interpreter charges every executed op a cycle cost under the
Spyre model of ktir_cpu/latency.py (categories :25-32, HardwareConfig
:34-80, per-core counters :90-126, per-op estimate LatencyTracker._estimate
:175-265, report :416-620).  The B200 backend does not execute ops one by
one, so the same charges are derived from the host trace instead: the tracer
visits every op of every core in the reference's order (scf.for bodies per
iteration, linalg.generic / tensor.generate bodies once on full-shape
operands, linalg.reduce combiners once per pairwise-fold round) and appends
one tape entry per op.  Memory ops are charged at 128-byte stick granularity
from the addresses they touch (rectangular: ktir_cpu/ops/memory_ops.py:492-502
and :406-436; indirect: data sticks of the gathered coordinates plus the
distinct sticks of every index view, :189-261 and :914-966).  Indirect
entries depend on index values, so they are resolved per call from the
host-side inputs; index tensors written by the same call are charged with
their values at call entry.

The report classes keep the reference's surface (``kernel_cycles``,
``kernel_time_us``, ``bottleneck``, ``per_core_summary``, ``roofline``,
``summary_dict``, ``str``) and accept the reference's own HardwareConfig.
Counters are accumulated in op order with the same arithmetic, so the
floating-point totals equal the reference's exactly.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Callable, Dict, List, Optional

import numpy as np

STICK = 128


class LatencyCategory(str, Enum):
    """Cost classes of ktir_cpu/latency.py:25-32 (string-valued)."""
    ZERO = "zero"
    MEMORY = "memory"
    COMPUTE_FLOAT = "compute_float"
    COMPUTE_TRANSCENDENTAL = "compute_transcendental"
    COMPUTE_INT = "compute_int"
    COMPUTE_MATMUL = "compute_matmul"
    COMM = "comm"

    def __str__(self) -> str:
        return self.value


@dataclass
class HardwareConfig:
    """Spyre model parameters, defaults of ktir_cpu/latency.py:34-80."""
    num_cores: int = 32
    clock_ghz: float = 1.0
    hbm_bandwidth_tb_s: float = 1.0
    ring_bandwidth_tb_s: float = 4.0
    simd_elements_per_cycle: int = 64
    systolic_flops_per_cycle: int = 2 * 64 * 64 * 64
    transcendental_penalty: int = 4

    @property
    def hbm_bytes_per_cycle_per_core(self) -> float:
        return self.hbm_bandwidth_tb_s * 1e12 / (self.clock_ghz * 1e9) / self.num_cores

    @property
    def ring_bytes_per_cycle(self) -> float:
        return self.ring_bandwidth_tb_s * 1e12 / (self.clock_ghz * 1e9)


# op -> category, as the reference registers them (ktir_cpu/dialects/*.py
# @register(..., latency_category=...)); every other op costs nothing
_FLOAT = ("arith.addf arith.subf arith.mulf arith.divf arith.remf arith.negf arith.absf "
          "arith.maxf arith.maximumf arith.maxnumf arith.minf arith.minimumf arith.minnumf "
          "arith.cmpf arith.cmpi arith.select math.absf math.absi math.ceil math.floor math.fma "
          "linalg.add linalg.generic")
_INT = ("arith.addi arith.subi arith.muli arith.divui arith.divsi arith.ceildivsi "
        "arith.floordivsi arith.remui arith.remsi arith.minsi arith.maxsi arith.minui "
        "arith.maxui arith.ceildivui arith.andi arith.ori arith.xori arith.shli arith.shrsi "
        "arith.shrui")
_TRANS = ("math.exp math.sqrt math.rsqrt math.log math.log2 math.log1p math.tanh math.sin "
          "math.cos math.erf math.powf")
CATEGORY: Dict[str, str] = {}
for _names, _cat in ((_FLOAT, "compute_float"), (_INT, "compute_int"),
                     (_TRANS, "compute_transcendental"),
                     ("linalg.matmul linalg.batch_matmul", "compute_matmul"),
                     ("ktdp.load ktdp.store", "memory"), ("ktdp.inter_tile_reduce", "comm")):
    for _n in _names.split():
        CATEGORY[_n] = _cat


def category(op_type: str) -> str:
    return CATEGORY.get(op_type, "zero")


@dataclass
class _TraceEntry:
    op_type: str
    cycles: float
    category: str


@dataclass
class CoreLatencyCounters:
    """Per-core counters (ktir_cpu/latency.py:90-126)."""
    memory_cycles: float = 0.0
    comm_cycles: float = 0.0
    total_bytes: int = 0
    flops_by_category: Dict[str, float] = field(default_factory=dict)
    cycles_by_category: Dict[str, float] = field(default_factory=dict)
    trace: Optional[List[_TraceEntry]] = None

    @property
    def compute_cycles(self) -> float:
        return sum(self.cycles_by_category.values())

    @property
    def total_cycles(self) -> float:
        return self.compute_cycles + self.memory_cycles + self.comm_cycles

    @property
    def total_flops(self) -> float:
        return sum(self.flops_by_category.values())

    def record(self, cat: str, cycles: float, op_type: str = "", flops: float = 0.0,
               nbytes: int = 0) -> None:
        if cat.startswith("compute_"):
            self.cycles_by_category[cat] = self.cycles_by_category.get(cat, 0.0) + cycles
            self.flops_by_category[cat] = self.flops_by_category.get(cat, 0.0) + flops
        elif cat == "memory":
            self.memory_cycles += cycles
        elif cat == "comm":
            self.comm_cycles += cycles
        self.total_bytes += nbytes
        if self.trace is not None:
            self.trace.append(_TraceEntry(op_type, cycles, cat))


@dataclass
class LatencyReport:
    """Kernel-level summary (ktir_cpu/latency.py:416-620)."""
    config: Any
    counters: Dict[int, CoreLatencyCounters]

    @property
    def kernel_cycles(self) -> float:
        if not self.counters:
            return 0.0
        return max(c.total_cycles for c in self.counters.values())

    @property
    def kernel_time_us(self) -> float:
        return self.kernel_cycles / (self.config.clock_ghz * 1e3)

    def _critical(self) -> CoreLatencyCounters:
        return max(self.counters.values(), key=lambda c: c.total_cycles)

    @property
    def bottleneck(self) -> str:
        if not self.counters:
            return "none"
        c = self._critical()
        parts = {"compute": c.compute_cycles, "memory": c.memory_cycles, "comm": c.comm_cycles}
        return max(parts, key=parts.get)

    def per_core_summary(self) -> List[Dict[str, Any]]:
        return [{"core_id": cid, "compute_cycles": c.compute_cycles,
                 "memory_cycles": c.memory_cycles, "comm_cycles": c.comm_cycles,
                 "total_cycles": c.total_cycles}
                for cid, c in sorted(self.counters.items())]

    def roofline(self) -> Dict[str, Any]:
        """Per-unit roofline of the critical-path core (systolic = matmul, simd = rest)."""
        if not self.counters:
            return {}
        crit = self._critical()
        clock = self.config.clock_ghz * 1e9
        elapsed = crit.total_cycles / clock
        peak_bw = self.config.hbm_bytes_per_cycle_per_core * clock
        ai = crit.total_flops / crit.total_bytes if crit.total_bytes > 0 else float("inf")
        peaks = {"systolic": self.config.systolic_flops_per_cycle * clock,
                 "simd": self.config.simd_elements_per_cycle * clock}
        cats = {"systolic": ("compute_matmul",),
                "simd": ("compute_float", "compute_transcendental", "compute_int")}
        flops = {u: sum(crit.flops_by_category.get(c, 0.0) for c in cats[u]) for u in peaks}
        units: Dict[str, Any] = {}
        for u, peak in peaks.items():
            achieved = flops[u] / elapsed if elapsed > 0 else 0.0
            ceiling = min(peak, peak_bw * ai)
            units[u] = {"achieved_gflops": achieved / 1e9, "ceiling_gflops": ceiling / 1e9,
                        "ridge_point": peak / peak_bw,
                        "efficiency": achieved / ceiling if ceiling > 0 else 0.0}
        dominant = max(peaks, key=lambda u: flops[u])
        if all(units[u]["achieved_gflops"] == 0.0 for u in units):
            dominant = "simd"
        return {"arithmetic_intensity": ai, "peak_bw_gb_s": peak_bw / 1e9,
                "dominant_unit": dominant, "efficiency": units[dominant]["efficiency"],
                "units": units}

    def summary_dict(self) -> Dict[str, Any]:
        return {"kernel_cycles": self.kernel_cycles, "kernel_time_us": self.kernel_time_us,
                "bottleneck": self.bottleneck, "num_cores": len(self.counters),
                "per_core": self.per_core_summary()}

    def __str__(self) -> str:
        bar = "=" * 60
        out = [bar, "KTIR Latency Estimation Report", bar,
               f"  Kernel cycles : {self.kernel_cycles:,.0f}",
               f"  Kernel time   : {self.kernel_time_us:.3f} us",
               f"  Bottleneck    : {self.bottleneck}",
               f"  Cores         : {len(self.counters)}", "-" * 60,
               f"  {'Core':>4}  {'Compute':>12}  {'Memory':>12}  {'Comm':>12}  {'Total':>12}",
               "-" * 60]
        for cid in sorted(self.counters):
            c = self.counters[cid]
            out.append(f"  {cid:>4}  {c.compute_cycles:>12.0f}  {c.memory_cycles:>12.0f}  "
                       f"{c.comm_cycles:>12.0f}  {c.total_cycles:>12.0f}")
        out.append(bar)
        if self.counters:
            crit = self._critical()
            if crit.total_flops > 0 or crit.total_bytes > 0:
                rf = self.roofline()
                ai = rf["arithmetic_intensity"]
                ai_s = f"{ai:.2f} FLOP/B" if ai != float("inf") else "inf (no memory traffic)"
                out += ["", "Roofline Analysis (critical-path core)", "-" * 60,
                        f"  Arithmetic intensity : {ai_s}",
                        f"  Peak bandwidth       : {rf['peak_bw_gb_s']:.2f} GB/s",
                        f"  Dominant unit        : {rf['dominant_unit']}",
                        f"  Efficiency           : {rf['efficiency']:.1%}  (dominant unit)", "",
                        f"  {'Unit':>10}  {'Achieved':>12}  {'Ceiling':>12}  {'Ridge':>10}  "
                        f"{'Eff':>7}",
                        f"  {'-' * 10}  {'-' * 12}  {'-' * 12}  {'-' * 10}  {'-' * 7}"]
                for u, d in rf["units"].items():
                    mark = " *" if u == rf["dominant_unit"] else "  "
                    out.append(f"{mark} {u:>10}  {d['achieved_gflops']:>10.2f} G  "
                               f"{d['ceiling_gflops']:>10.2f} G  {d['ridge_point']:>8.1f} F/B  "
                               f"{d['efficiency']:>6.1%}")
                out.append(bar)
        return "\n".join(out)


# ---------------------------------------------------------------------------
# stick counting
# ---------------------------------------------------------------------------

def _is_row_major(shape, strides) -> bool:
    want = 1
    for n, s in zip(reversed(shape), reversed(strides)):
        if s != want:
            return False
        want *= n
    return True


def rect_sticks(byte_base: int, shape, strides, itemsize: int) -> int:
    """Distinct 128-byte sticks touched by a strided box starting at byte_base."""
    shape = tuple(int(s) for s in shape)
    if _is_row_major(shape, strides):
        n = int(np.prod(shape)) if shape else 1
        return -(-(byte_base + n * itemsize) // STICK) - byte_base // STICK
    if any(s == 0 for s in shape):
        return 0
    off = np.zeros((), np.int64)
    for n, s in zip(shape, strides):
        off = np.add.outer(off, np.arange(n, dtype=np.int64) * int(s))
    return coord_sticks(byte_base, off.reshape(-1), itemsize)


def coord_sticks(byte_base: int, offsets: np.ndarray, itemsize: int) -> int:
    if offsets.size == 0:
        return 0
    return int(np.unique((byte_base + offsets.astype(np.int64) * itemsize) // STICK).size)


# ---------------------------------------------------------------------------
# tape: what the tracer records; replayed per call into counters
# ---------------------------------------------------------------------------

class LatencyTape:
    """Per-core op records taken by the tracer.

    Entries are (op_type, category, n) where n is the element count (compute),
    the (m, n, k) triple (matmul) or the stick count (memory); an indirect
    memory op stores its access descriptor instead and is resolved per call.
    """

    def __init__(self) -> None:
        self.cores: Dict[int, List[tuple]] = {}
        self.cur: Optional[List[tuple]] = None

    def begin_core(self, cid: int) -> None:
        self.cur = self.cores.setdefault(cid, [])

    def add(self, op_type: str, cat: str, arg: Any = None) -> None:
        self.cur.append((op_type, cat, arg))

    def has_indirect(self) -> bool:
        return any(isinstance(e[2], IndirectAccess) for es in self.cores.values() for e in es)

    def report(self, config: Any, trace: bool = False,
               read_index: Optional[Callable[[int, np.ndarray, np.dtype], np.ndarray]] = None
               ) -> LatencyReport:
        """Replay the tape under `config`.  `read_index(byte_addr, addrs, dtype)`
        returns index-tensor values at the given byte addresses (call inputs)."""
        bw = config.hbm_bytes_per_cycle_per_core
        simd = config.simd_elements_per_cycle
        counters: Dict[int, CoreLatencyCounters] = {}
        for cid, entries in self.cores.items():
            c = CoreLatencyCounters(trace=[] if trace else None)
            counters[cid] = c
            for op_type, cat, arg in entries:
                if cat == "zero":
                    c.record("zero", 0.0, op_type)
                elif cat == "memory":
                    sticks = arg.sticks(read_index) if isinstance(arg, IndirectAccess) else arg
                    nbytes = sticks * STICK
                    c.record("memory", nbytes / bw if bw > 0 else 0.0, op_type, nbytes=nbytes)
                elif cat == "compute_matmul":
                    m, n, k = arg
                    flops = 2.0 * m * n * k
                    c.record(cat, flops / config.systolic_flops_per_cycle, op_type, flops=flops)
                elif cat == "compute_transcendental":
                    c.record(cat, (arg / simd) * config.transcendental_penalty, op_type,
                             flops=float(arg))
                elif cat == "compute_float":
                    c.record(cat, arg / simd, op_type, flops=float(arg))
                elif cat == "compute_int":
                    if arg <= 1:
                        c.record(cat, 0.0, op_type, flops=0.0)
                    else:
                        c.record(cat, arg / simd, op_type, flops=float(arg))
                elif cat == "comm":
                    if arg is None:
                        raise RuntimeError("_comm_size: comm op result must be a Tile, "
                                           "got NoneType")
                    rb = config.ring_bytes_per_cycle
                    c.record("comm", arg / rb if rb > 0 else 0.0, op_type, nbytes=int(arg))
                else:
                    raise NotImplementedError(f"latency category {cat}")
        return LatencyReport(config=config, counters=counters)


class IndirectAccess:
    """An indirect load/store whose stick count depends on index values."""

    def __init__(self, iat, store: bool) -> None:
        self.iat = iat
        self.store = store

    def sticks(self, read_index) -> int:
        from .affine import eval_expr
        from .trace import bpe
        iat = self.iat
        pts = iat.vss.enumerate_array(iat.shape)
        if iat.vso is not None and len(pts):
            keys = np.stack([np.broadcast_to(np.asarray(k, np.int64), (pts.shape[0],))
                             for k in iat.vso.eval(list(pts.T))], axis=1)
            pts = pts[np.lexsort(keys.T[::-1])]
        n = pts.shape[0]
        if n == 0:
            return 0
        cols = [pts[:, i].astype(np.int64) for i in range(pts.shape[1])]
        for i, v in iat.consts.items():
            cols[i] = np.full(n, v, np.int64)

        def ev(e):
            return np.broadcast_to(np.asarray(eval_expr(e, cols, (), iat.refs), np.int64), (n,))
        par = iat.parent
        off = np.zeros(n, np.int64)
        view_addrs: Dict[int, List[np.ndarray]] = {}
        for k, d in enumerate(iat.dims):
            if d["kind"] == "direct":
                off = off + ev(d["expr"]) * par.strides[k]
                continue
            view = iat.views[d["view"]]
            vb = bpe(view.dtype)
            io = np.zeros(n, np.int64)
            for e, s in zip(d["exprs"], view.strides):
                io = io + ev(e) * s
            addrs = view.byte_address + io * vb
            view_addrs.setdefault(d["view"], []).append(addrs)
            vals = read_index(addrs, view.dtype).astype(np.int64)
            off = off + vals * par.strides[k]
        data = coord_sticks(par.byte_address, off, bpe(par.dtype))
        idx = 0
        for addrs in view_addrs.values():
            a = np.concatenate(addrs)
            idx += int(np.unique(a // STICK).size)
        return data + idx
