"""Lowering of a traced KTIR call onto device programs.

The trace (:mod:`ktir_cpu_b200.trace`) is a dataflow graph of tile nodes plus
an ordered list of stores per core.  This module turns it into a Plan: a
short list of launches of the library's kernels.

Fused programs, tried in order; each must account for every store:

  gather_rmw  every store is an indirect row scatter whose value is an
              elementwise function of the indirect gather through the same
              access tile (the read-modify-write pattern).  One count pass +
              one apply pass reproduce the reference's unit-by-unit result.
  gemm        every store is truncf(sum_k extf(A_k) @ extf(B_k)) over a
              K sweep, the stores tile C = A @ B exactly -> tcgen05 GEMM.
  attention   the attention rewrite replaced the online-softmax loop by a
              single node -> tcgen05 flash attention.
  softmax     every store is a row softmax of a rectangular row-block load.
  elementwise every store is an elementwise DAG of rectangular loads.

Stores of different units must not write what other units read or write
(checked on element intervals); otherwise, and for everything else, the
generic executor runs the graph core by core, node by node, in program
order — the reference's sequential semantics — with kernels for loads,
elementwise bytecode, tree reductions, CUDA-core matmuls and stores.
"""

from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import runtime as R
from .affine import BoxSet, linearize
from .trace import Const, CoordTarget, IATV, IndirectTarget, Node, RectTarget, Store, Trace

# ---------------------------------------------------------------------------
# elementwise bytecode compiler
# ---------------------------------------------------------------------------

OP = dict(NOP=0, LD=1, ST=2, IMM=3, IOTA=4, CAST=5, BITCAST=6,
          FADD=10, FSUB=11, FMUL=12, FDIV=13, FMOD=14, FMAXNUM=15, FMINNUM=16, FMAXIMUM=17,
          FMINIMUM=18, FPOW=19, FNEG=20, FABS=21, FEXP=22, FSQRT=23, FRSQRT=24, FLOG=25,
          FLOG2=26, FLOG1P=27, FTANH=28, FSIN=29, FCOS=30, FCEIL=31, FFLOOR=32, FERF=33,
          FFMA=34, FCMP=35, SELECT=36, IADD=40, ISUB=41, IMUL=42, IFLOORDIV=43, IMOD=44,
          ITRUNCDIV=45, ITRUNCREM=46, ICEILDIV=47, IAND=48, IOR=49, IXOR=50, ISHL=51,
          ISHR=52, ISHRU=53, IMAX=54, IMIN=55, INEG=56, IABS=57, ICMP=58)

_FBIN = {"add": "FADD", "sub": "FSUB", "mul": "FMUL", "div": "FDIV", "fmod": "FMOD",
         "fmax": "FMAXNUM", "fmin": "FMINNUM", "maximum": "FMAXIMUM", "minimum": "FMINIMUM",
         "pow": "FPOW"}
_IBIN = {"add": "IADD", "sub": "ISUB", "mul": "IMUL", "floordiv": "IFLOORDIV", "mod": "IMOD",
         "truncdiv": "ITRUNCDIV", "truncrem": "ITRUNCREM", "ceildiv": "ICEILDIV", "and": "IAND",
         "or": "IOR", "xor": "IXOR", "shl": "ISHL", "shr": "ISHR", "shru": "ISHRU",
         "maximum": "IMAX", "minimum": "IMIN", "fmax": "IMAX", "fmin": "IMIN"}
_FUN = {"neg": "FNEG", "abs": "FABS", "exp": "FEXP", "sqrt": "FSQRT", "rsqrt": "FRSQRT",
        "log": "FLOG", "log2": "FLOG2", "log1p": "FLOG1P", "tanh": "FTANH", "sin": "FSIN",
        "cos": "FCOS", "ceil": "FCEIL", "floor": "FFLOOR", "erf": "FERF"}
FPRED = {"false": 0, "oeq": 1, "ogt": 2, "oge": 3, "olt": 4, "ole": 5, "one": 6, "ord": 7,
         "ueq": 8, "ugt": 9, "uge": 10, "ult": 11, "ule": 12, "une": 13, "uno": 14, "true": 15}
IPRED = {"eq": 0, "ne": 1, "slt": 2, "sle": 3, "sgt": 4, "sge": 5, "ult": 6, "ule": 7,
         "ugt": 8, "uge": 9}
COMBINER = {"arith.addf": "FADD", "arith.mulf": "FMUL", "arith.maxnumf": "FMAXNUM",
            "arith.minnumf": "FMINNUM", "arith.maximumf": "FMAXIMUM", "arith.maxf": "FMAXIMUM",
            "arith.minimumf": "FMINIMUM", "arith.minf": "FMINIMUM", "arith.subf": "FSUB",
            "arith.divf": "FDIV", "arith.addi": "IADD", "arith.muli": "IMUL",
            "arith.maxsi": "IMAX", "arith.minsi": "IMIN", "arith.andi": "IAND",
            "arith.ori": "IOR", "arith.xori": "IXOR"}


def is_float(dt) -> bool:
    return np.dtype(dt).kind == "f"


class EwBuilder:
    """Compiles elementwise DAGs into KtirInstr lists over a shared view table."""

    def __init__(self, max_views: int = R.MAX_VIEWS):
        self.code: List[Tuple] = []
        self.views: List[Any] = []          # opaque view keys, resolved by the caller
        self.view_index: Dict[Any, int] = {}
        self.max_views = max_views
        self.free = list(range(R.NREG))[::-1]
        self.reg_of: Dict[int, Tuple[int, np.dtype]] = {}
        self.uses: Dict[int, int] = {}

    def view(self, key) -> int:
        if key not in self.view_index:
            if len(self.views) >= self.max_views:
                raise NotImplementedError("elementwise program needs too many views")
            self.view_index[key] = len(self.views)
            self.views.append(key)
        return self.view_index[key]

    def alloc(self) -> int:
        if not self.free:
            raise NotImplementedError("elementwise program needs too many registers")
        return self.free.pop()

    def release(self, r: int) -> None:
        self.free.append(r)

    def emit(self, op, dst=0, a=0, b=0, c=0, dt=0, aux=0, imm=0):
        if len(self.code) >= R.MAX_INSTR:
            raise NotImplementedError("elementwise program too long")
        self.code.append((OP[op], dst, a, b, c, dt, aux, 0, imm))

    def imm(self, value, dt) -> int:
        r = self.alloc()
        code = R.dtype_code(dt)
        if is_float(dt):
            self.emit("IMM", r, dt=code, imm=R.double_bits(float(value)))
        else:
            self.emit("IMM", r, dt=code, imm=int(value))
        return r

    def cast(self, r: int, src, dst) -> int:
        src, dst = np.dtype(src), np.dtype(dst)
        if src == dst:
            return r
        o = self.alloc()
        self.emit("CAST", o, r, dt=R.dtype_code(dst), aux=R.dtype_code(src))
        self.release(r)
        return o

    def fill(self, instrs) -> Tuple[Any, int]:
        arr = (R.KtirInstr * R.MAX_INSTR)()
        for i, t in enumerate(self.code):
            arr[i] = R.KtirInstr(*t)
        return arr, len(self.code)


def compile_ew(b: EwBuilder, root, leaf: Callable[[Node], Optional[Tuple[str, Any]]]) -> Tuple[int, np.dtype]:
    """Emit code computing `root`; returns (register, dtype).

    `leaf(node)` returns ("view", key) for nodes loaded through a view,
    ("imm", (value, dtype)) for immediates, or None to compile the node here.
    """
    memo: Dict[int, Tuple[int, np.dtype]] = {}
    # count uses inside this DAG to know when a register can be recycled
    uses: Dict[int, int] = {}

    def count(n):
        if isinstance(n, Const):
            return
        uses[n.id] = uses.get(n.id, 0) + 1
        if uses[n.id] > 1:
            return
        if leaf(n) is None and n.kind == "ew":
            for i in n.ins:
                count(i)
        elif leaf(n) is None and n.kind in ("splat",):
            count(n.ins[0])

    count(root)

    def operand(x, want) -> int:
        if isinstance(x, Const):
            return b.imm(x.value, want)
        r, dt = get(x)
        if uses[x.id] > 1:
            # keep the shared value; work on a copy when converting
            uses[x.id] -= 1
            if np.dtype(dt) != np.dtype(want):
                o = b.alloc()
                b.emit("CAST", o, r, dt=R.dtype_code(want), aux=R.dtype_code(dt))
                return o
            o = b.alloc()
            b.emit("CAST", o, r, dt=R.dtype_code(want), aux=R.dtype_code(dt))
            return o
        uses[x.id] -= 1
        return b.cast(r, dt, want)

    def get(n) -> Tuple[int, np.dtype]:
        if n.id in memo:
            return memo[n.id]
        lf = leaf(n)
        if lf is not None:
            kind, payload = lf
            if kind == "view":
                r = b.alloc()
                b.emit("LD", r, aux=b.view(payload))
                res = (r, n.dtype)
            elif kind == "iota":
                r = b.alloc()
                b.emit("IOTA", r, aux=payload, dt=R.I64)
                res = (r, np.dtype(np.int64))
            else:
                val, dt = payload
                res = (b.imm(val, dt), np.dtype(dt))
        elif n.kind == "splat":
            res = get(n.ins[0])
        elif n.kind == "ew":
            res = (emit_ew(n), n.dtype)
        else:
            raise NotImplementedError(f"cannot inline {n.kind} into an elementwise program")
        memo[n.id] = res
        return res

    def emit_ew(n: Node) -> int:
        op = n.attrs["op"]
        dt = n.dtype
        code = R.dtype_code(dt)
        if op == "cast":
            x = n.ins[0]
            src = x.dtype if isinstance(x, Node) else x.dtype
            r = operand(x, src)
            return b.cast(r, src, dt) if np.dtype(src) != dt else r
        if op == "bitcast":
            r = operand(n.ins[0], n.ins[0].dtype)
            o = b.alloc()
            b.emit("BITCAST", o, r, dt=code)
            b.release(r)
            return o
        if op == "cmp":
            a, c = n.ins
            ad = a.dtype if isinstance(a, Node) else a.dtype
            cd = c.dtype if isinstance(c, Node) else c.dtype
            cdt = np.result_type(ad, cd)
            if cdt == np.float64:
                cdt = np.dtype(np.float32)
            ra, rc = operand(a, cdt), operand(c, cdt)
            o = b.alloc()
            if is_float(cdt):
                b.emit("FCMP", o, ra, rc, dt=R.BOOL, aux=FPRED[n.attrs["pred"]])
            else:
                b.emit("ICMP", o, ra, rc, dt=R.BOOL, aux=IPRED[n.attrs["pred"]])
            b.release(ra)
            b.release(rc)
            return o
        if op == "select":
            cnd, t, f = n.ins
            rc = operand(cnd, np.bool_)
            rt, rf = operand(t, dt), operand(f, dt)
            o = b.alloc()
            b.emit("SELECT", o, rc, rt, rf, dt=code)
            for r in (rc, rt, rf):
                b.release(r)
            return o
        if op == "fma":
            rs = [operand(x, dt) for x in n.ins]
            o = b.alloc()
            b.emit("FFMA", o, *rs, dt=code)
            for r in rs:
                b.release(r)
            return o
        if is_float(dt):
            if op in _FUN:
                r = operand(n.ins[0], dt)
                o = b.alloc()
                b.emit(_FUN[op], o, r, dt=code)
                b.release(r)
                return o
            if op in _FBIN:
                ra, rb = operand(n.ins[0], dt), operand(n.ins[1], dt)
                o = b.alloc()
                b.emit(_FBIN[op], o, ra, rb, dt=code)
                b.release(ra)
                b.release(rb)
                return o
        else:
            if op == "neg":
                r = operand(n.ins[0], dt)
                o = b.alloc()
                b.emit("INEG", o, r, dt=code)
                b.release(r)
                return o
            if op == "abs":
                r = operand(n.ins[0], dt)
                o = b.alloc()
                b.emit("IABS", o, r, dt=code)
                b.release(r)
                return o
            if op in _IBIN:
                ra, rb = operand(n.ins[0], dt), operand(n.ins[1], dt)
                o = b.alloc()
                b.emit(_IBIN[op], o, ra, rb, dt=code)
                b.release(ra)
                b.release(rb)
                return o
        raise NotImplementedError(f"elementwise op {op} on {dt}")

    return get(root)


def program(b: EwBuilder, shape, n_units: int, unit_cols: int,
            view_fn: Callable[[Any], R.KtirView], contiguous: bool = False) -> R.KtirEwProgram:
    p = R.KtirEwProgram()
    p.rank = len(shape)
    p.n_views = len(b.views)
    p.n_instr = len(b.code)
    p.n_units = n_units
    p.unit_cols = unit_cols
    p.contiguous = 1 if contiguous else 0
    p.numel = int(np.prod(shape)) if shape else 1
    for i, s in enumerate(shape):
        p.shape[i] = int(s)
    for i, key in enumerate(b.views):
        p.view[i] = view_fn(key)
    for i, t in enumerate(b.code):
        p.code[i] = R.KtirInstr(*t)
    return p


def mkview(slot, dtype, off, strides, unit_col=-1, pad=0) -> R.KtirView:
    v = R.KtirView()
    v.slot = slot
    v.dtype = R.dtype_code(dtype)
    v.unit_col = unit_col
    v.pad = pad
    v.off = int(off)
    for i, s in enumerate(strides):
        v.stride[i] = int(s)
    return v


def dense_strides(shape) -> Tuple[int, ...]:
    st, acc = [], 1
    for s in reversed(shape):
        st.append(acc)
        acc *= s
    return tuple(reversed(st))


def align_strides(strides, shape_in, shape_out) -> Tuple[int, ...]:
    """Right-align a view's strides to an iteration space (NumPy broadcasting)."""
    nd = len(shape_out)
    off = nd - len(shape_in)
    out = [0] * nd
    for i, (s, n) in enumerate(zip(strides, shape_in)):
        out[off + i] = 0 if (n == 1 and shape_out[off + i] != 1) else s
    return tuple(out)


# ---------------------------------------------------------------------------
# plan
# ---------------------------------------------------------------------------

@dataclass
class Launch:
    fn: Callable[..., None]       # fn(bufs, stream) issues the launch
    kind: str
    kernels: int = 1
    meta: Dict[str, Any] = field(default_factory=dict)


@dataclass
class Plan:
    kind: str
    launches: List[Launch]
    slots: List[int]                              # call buffer index -> slot
    arena_bytes: int = 0
    status_check: bool = False
    host_arrays: List[np.ndarray] = field(default_factory=list)
    device_arrays: List[Any] = field(default_factory=list)
    scratch: Dict[str, Any] = field(default_factory=dict)
    info: Dict[str, Any] = field(default_factory=dict)

    @property
    def kernel_launches(self) -> int:
        return sum(l.kernels for l in self.launches)

    @property
    def collective(self) -> bool:
        """Whether a launch exchanges data with other ranks (NCCL calls, which
        stay out of CUDA graphs)."""
        return any(l.kind in COLLECTIVE_KINDS for l in self.launches)


# launch kinds that are NCCL exchanges between ranks
COLLECTIVE_KINDS = {"reduce_scatter_counts", "kv_ring"}


class DeviceData:
    """Owns the device-side copies of host index tables of a plan."""

    def __init__(self, device):
        import torch
        self.torch = torch
        self.device = device
        self.keep: List[Any] = []

    def i64(self, arr: np.ndarray) -> int:
        t = self.torch.from_numpy(np.ascontiguousarray(arr, dtype=np.int64)).to(self.device)
        self.keep.append(t)
        return t.data_ptr()

    def zeros_i32(self, n: int) -> Any:
        t = self.torch.zeros(max(1, int(n)), dtype=self.torch.int32, device=self.device)
        self.keep.append(t)
        return t

    def bytes(self, n: int) -> Any:
        t = self.torch.zeros(max(16, int(n)), dtype=self.torch.uint8, device=self.device)
        self.keep.append(t)
        return t


# ---------------------------------------------------------------------------
# helpers over the trace
# ---------------------------------------------------------------------------

def _interval(buf_off: int, shape, strides) -> Tuple[int, int]:
    lo = hi = buf_off
    for n, s in zip(shape, strides):
        if n <= 0:
            return (buf_off, buf_off - 1)
        if s >= 0:
            hi += (n - 1) * s
        else:
            lo += (n - 1) * s
    return lo, hi


def _target_interval(t) -> Tuple[int, Tuple[int, int]]:
    if isinstance(t, RectTarget):
        return t.buf.index, _interval(t.off, t.shape, t.strides)
    if isinstance(t, CoordTarget):
        if t.offsets.size == 0:
            return t.buf.index, (0, -1)
        return t.buf.index, (t.off + int(t.offsets.min()), t.off + int(t.offsets.max()))
    raise TypeError(t)


def _load_interval(n: Node) -> Tuple[int, Tuple[int, int]]:
    a = n.attrs
    if a["mode"] == "rect":
        return a["buf"].index, _interval(a["off"], n.shape, a["strides"])
    if a["mode"] == "coords":
        o = a["offsets"]
        if o.size == 0:
            return a["buf"].index, (0, -1)
        return a["buf"].index, (a["off"] + int(o.min()), a["off"] + int(o.max()))
    return a["buf"].index, (0, 1 << 62)


def _leaves(root: Node) -> List[Node]:
    seen, out, stack = set(), [], [root]
    while stack:
        n = stack.pop()
        if not isinstance(n, Node) or n.id in seen:
            continue
        seen.add(n.id)
        if n.kind == "load":
            out.append(n)
        for i in n.ins:
            stack.append(i)
    return out


def _overlap(a: Tuple[int, int], b: Tuple[int, int]) -> bool:
    return a[0] <= b[1] and b[0] <= a[1]


def units_independent(items: Sequence[Tuple[List[Tuple[int, Tuple[int, int]]],
                                            List[Tuple[int, Tuple[int, int]]]]]) -> bool:
    """items[u] = (reads, writes); no unit may write what another reads or writes."""
    by_buf: Dict[int, List[Tuple[int, int, int, bool]]] = {}
    for u, (reads, writes) in enumerate(items):
        for buf, iv in reads:
            by_buf.setdefault(buf, []).append((iv[0], iv[1], u, False))
        for buf, iv in writes:
            by_buf.setdefault(buf, []).append((iv[0], iv[1], u, True))
    for evs in by_buf.values():
        if not any(w for *_, w in evs):
            continue
        evs.sort()
        # sweep: any overlapping pair from different units with at least one write
        active: List[Tuple[int, int, bool]] = []
        for lo, hi, u, w in evs:
            active = [x for x in active if x[0] >= lo]
            for ahi, au, aw in active:
                if au != u and (aw or w):
                    return False
            active.append((hi, u, w))
    return True


# ---------------------------------------------------------------------------
# the lowering entry point
# ---------------------------------------------------------------------------

def core_range(rank: int, world: int, n_cores: int) -> Tuple[int, int]:
    """Contiguous block of cores owned by `rank` when a grid is split across `world` GPUs."""
    return (rank * n_cores) // world, ((rank + 1) * n_cores) // world


def row_shard(rank: int, world: int, n_rows: int) -> Tuple[int, int, int]:
    """(first row, end row, chunk) of the table rows `rank` owns in a split
    gather-RMW: equal chunks of ceil(n_rows / world) rows, the last ones cut
    at n_rows, which is the layout a reduce-scatter of the per-row counts
    (padded to chunk * world entries) leaves on each rank."""
    chunk = -(-n_rows // world)
    return min(n_rows, rank * chunk), min(n_rows, (rank + 1) * chunk), chunk


class Lowerer:
    """Lower one traced call.  With `shard=(rank, world, group)` only the stores
    of this rank's contiguous core range are lowered (the grid is split across
    GPUs); programs that need an exchange between shards get a collective."""

    def __init__(self, trace: Trace, device, slots: Dict[int, int], shard=None):
        self.trace = trace
        self.device = device
        self.slots = slots            # buffer index -> slot
        self.dev = DeviceData(device)
        self.shard = shard

    def lower(self) -> Plan:
        stores = self.trace.stores
        self.all_stores = stores
        if self.shard is not None:
            rank, world = self.shard[0], self.shard[1]
            nx, ny, nz = self.trace.grid
            c0, c1 = core_range(rank, world, nx * ny * nz)
            stores = [s for s in stores if c0 <= s.core < c1]
        for matcher in (self.match_gather_rmw, self.match_gemm, self.match_attention,
                        self.match_softmax, self.match_elementwise):
            plan = matcher(stores)
            if plan is not None:
                plan.device_arrays = self.dev.keep
                return self.finish(plan)
        plan = GenericExecutor(self).build()
        plan.device_arrays = self.dev.keep
        return self.finish(plan)

    def finish(self, plan: Plan) -> Plan:
        """Record which call buffers the plan may write (others need no download)."""
        written = set()
        for s in self.trace.stores:
            t = s.target
            if isinstance(t, IndirectTarget):
                b = self.trace.space.find(t.iat.parent.byte_address)
                written.add(b.index)
            else:
                written.add(t.buf.index)
        plan.info["written"] = written
        plan.info["overwritten"] = self._overwritten()
        return plan

    def _overwritten(self) -> set:
        """Buffers the call never reads and whose every element it stores:
        their contents before the call cannot show, so they need no upload."""
        if self.shard is not None:
            return set()
        sp = self.trace.space
        read = set()

        def views_of(iat):
            for v in [iat.parent] + list(iat.views):
                b = sp.find(v.byte_address)
                if b is not None:
                    read.add(b.index)
        for n in self.trace.nodes:
            if n.kind == "load":
                read.add(n.attrs["buf"].index)
                if n.attrs["mode"] == "indirect":
                    views_of(n.attrs["iat"])
        masks: Dict[int, np.ndarray] = {}
        for s in self.trace.stores:
            t = s.target
            if isinstance(t, IndirectTarget):
                views_of(t.iat)
                continue
            b = t.buf
            if b.index in read:
                continue
            m = masks.get(b.index)
            if m is None:
                if b.numel > (1 << 28):
                    read.add(b.index)
                    continue
                m = masks[b.index] = np.zeros(b.numel, dtype=bool)
            if isinstance(t, RectTarget):
                offs = np.full((), t.off, np.int64)
                for n_, st in zip(t.shape, t.strides):
                    offs = np.add.outer(offs, np.arange(n_, dtype=np.int64) * st)
                offs = offs.reshape(-1)
            else:
                offs = t.off + np.asarray(t.offsets, np.int64)
            m[offs[(offs >= 0) & (offs < b.numel)]] = True
        return {i for i, m in masks.items() if i not in read and bool(m.all())}

    # -- gather -> f -> scatter ----------------------------------------------------
    def match_gather_rmw(self, stores: List[Store]) -> Optional[Plan]:
        if self.shard is not None:
            # every unit's indices are needed to apply the owned rows; the
            # local units only decide this shard's share of the counts
            full = self._gather_rmw_desc(self.all_stores)
            local = self._gather_rmw_desc(stores) if stores else None
            if full is None or (stores and local is None):
                return None
            return self._gather_rmw_plan(full, local)
        d = self._gather_rmw_desc(stores)
        return None if d is None else self._gather_rmw_plan(d, None)

    def _gather_rmw_desc(self, stores: List[Store]):
        if not stores or not all(isinstance(s.target, IndirectTarget) for s in stores):
            return None
        table_buf = None
        units = []
        fdag = None
        for s in stores:
            iat = s.target.iat
            loads = _leaves(s.value)
            if len(loads) != 1 or loads[0].attrs["mode"] != "indirect":
                return None
            ld = loads[0]
            if ld.attrs["iat"] is not iat:
                return None
            form = _row_gather_form(iat)
            if form is None:
                return None
            if s.value.shape != ld.shape or not _elementwise_only(s.value, ld):
                return None
            buf = ld.attrs["buf"]
            if table_buf is None:
                table_buf = buf
            elif buf is not table_buf:
                return None
            units.append((form, ld, s.value))
            if fdag is None:
                fdag = (ld, s.value)
        (R_, C_, row_stride, idx_view, idx_elem), ld0, v0 = units[0]
        del idx_elem
        if any(u[0][:3] != (R_, C_, row_stride) for u in units):
            return None
        if table_buf.dtype != np.float16 or v0.dtype != np.float16:
            return None
        idx_buf = _resolve_buffer(self.trace, idx_view)
        if idx_buf is None or idx_buf is table_buf:
            return None
        starts = [u[0][4] for u in units]
        steps = np.diff(starts) if len(starts) > 1 else np.array([0])
        if len(starts) > 1 and not np.all(steps == steps[0]):
            return None
        step = int(steps[0]) if len(starts) > 1 else 0
        # compile f with view 0 = gathered element, view 1 = result
        bld = EwBuilder()
        ld_key, st_key = ("g",), ("s",)

        def leaf(n):
            return ("view", ld_key) if n is ld0 else (
                ("imm", (n.attrs["value"], n.dtype)) if n.kind == "const" else None)
        b_leaf = leaf
        bld.view(ld_key)
        bld.view(st_key)
        r, dt = compile_ew(bld, v0, b_leaf)
        bld.emit("ST", 0, r, dt=R.dtype_code(dt), aux=1)
        d = R.KtirGatherRmwDesc()
        d.table_slot = self.slots[table_buf.index]
        d.idx_slot = self.slots[idx_buf.index]
        d.idx_dtype = R.dtype_code(idx_buf.dtype)
        d.n_units = len(units)
        d.unit_len = R_
        d.row_len = C_
        d.table_off = ld0.attrs["off"]
        d.row_stride = row_stride
        d.idx_off = starts[0]
        d.idx_unit_stride = step
        d.f = program(bld, (1,), 1, 0, lambda k: mkview(0, np.float16, 0, (0,)))
        n_rows = -(-table_buf.numel // row_stride)
        return d, n_rows, len(units), R_, C_

    def _gather_rmw_plan(self, full, local) -> Plan:
        """One ktir_gather_rmw launch (count pass, then apply pass).  A split
        call owns a contiguous range of table rows (equal chunks, row_shard)
        instead of its cores' units: whether a row is applied, and how often,
        depends on every unit that names it, so each rank counts over every
        unit's indices (1 MiB of int32 for the benchmark's 262,144) but only
        the rows it owns, and applies those.  No counts cross GPUs; the index
        tensor is read by every rank.  `local` (this rank's own units) does
        not change the plan."""
        del local
        d, n_rows, n_units, R_, C_ = full
        counts = self.dev.zeros_i32(n_rows)
        if self.shard is not None:
            rank, world, _ = self.shard
            r0, r1, _ = row_shard(rank, world, n_rows)
            d.phases = 0
            # row_hi 0 would mean every row: an empty range is [n_rows, n_rows)
            d.row_lo, d.row_hi = (r0, r1) if r1 > r0 else (n_rows, n_rows)
        lib = R.load_library()
        cptr = C.c_void_p(counts.data_ptr())

        def run(bufs, stream, status):
            R.check(lib.ktir_gather_rmw(C.byref(d), C.byref(bufs), cptr, n_rows,
                                        C.c_void_p(status), stream), "ktir_gather_rmw")
        launches = [Launch(run, "gather_rmw", 2)]
        plan = Plan("gather_rmw", launches, [], status_check=True)
        plan.scratch["counts"] = counts
        plan.info.update(units=n_units, unit_len=R_, row_len=C_, idx_elems=n_units * R_,
                         table_rows=n_rows)
        return plan

    # -- GEMM / attention are filled in by the tensor-core modules ---------------------
    def match_gemm(self, stores):
        from .tc import match_gemm
        return match_gemm(self, stores)

    def match_attention(self, stores):
        from .tc import match_attention
        return match_attention(self, stores)

    # -- row softmax --------------------------------------------------------------------
    def match_softmax(self, stores: List[Store]) -> Optional[Plan]:
        if not stores:
            return None
        units = []
        compute_f16 = None
        for s in stores:
            t = s.target
            if not isinstance(t, RectTarget) or len(t.shape) != 2 or t.strides[1] != 1:
                return None
            m = _softmax_form(s.value)
            if m is None:
                return None
            ld, cf16 = m
            if ld.shape != t.shape or ld.attrs["strides"][1] != 1:
                return None
            if compute_f16 is None:
                compute_f16 = cf16
            if cf16 != compute_f16 or t.dtype != np.float16 or ld.dtype != np.float16:
                return None
            units.append((ld, t))
        ld0, t0 = units[0]
        rows, cols = t0.shape
        if any(u[1].shape != (rows, cols) or u[0].attrs["buf"] is not ld0.attrs["buf"] or
               u[1].buf is not t0.buf or u[0].attrs["strides"][0] != ld0.attrs["strides"][0] or
               u[1].strides[0] != t0.strides[0] for u in units):
            return None
        if cols < 64 or cols & (cols - 1) or cols > 4096:
            return None
        items = [([_load_interval(ld)], [_target_interval(t)]) for ld, t in units]
        if not units_independent(items):
            return None
        table = np.array([[ld.attrs["off"], t.off] for ld, t in units], dtype=np.int64)
        if np.any(table % 8) or ld0.attrs["strides"][0] % 8 or t0.strides[0] % 8:
            return None
        d = R.KtirSoftmaxDesc()
        d.rows, d.cols, d.n_units, d.unit_cols = rows, cols, len(units), 2
        # units that are consecutive row blocks of both tensors become one
        # affine row range: the kernel then needs no per-unit table
        s_in, s_out = ld0.attrs["strides"][0], t0.strides[0]
        u = np.arange(len(units), dtype=np.int64)
        affine = bool(np.all(table[:, 0] == table[0, 0] + u * rows * s_in) and
                      np.all(table[:, 1] == table[0, 1] + u * rows * s_out))
        d.compute_f16 = 1 if compute_f16 else 0
        d.pad = int(os.environ.get("KTIR_SOFTMAX_ROWS_PER_WARP", "0"))
        if affine:
            d.rows, d.n_units = rows * len(units), 1
            d.in_ = mkview(self.slots[ld0.attrs["buf"].index], np.float16, table[0, 0], (s_in, 1))
            d.out = mkview(self.slots[t0.buf.index], np.float16, table[0, 1], (s_out, 1))
        else:
            d.in_ = mkview(self.slots[ld0.attrs["buf"].index], np.float16, 0, (s_in, 1), unit_col=0)
            d.out = mkview(self.slots[t0.buf.index], np.float16, 0, (s_out, 1), unit_col=1)
        ut = self.dev.i64(table)
        lib = R.load_library()
        desc = d

        def run(bufs, stream, status):
            R.check(lib.ktir_softmax_rows(C.byref(desc), C.byref(bufs), C.c_void_p(ut), stream),
                    "ktir_softmax_rows")
        plan = Plan("softmax", [Launch(run, "softmax")], [])
        plan.info.update(rows=rows * len(units), cols=cols)
        return plan

    # -- elementwise ---------------------------------------------------------------------
    def match_elementwise(self, stores: List[Store]) -> Optional[Plan]:
        if not stores:
            return None
        groups: Dict[Any, List[Tuple[Store, List[Node]]]] = {}
        for s in stores:
            if not isinstance(s.target, RectTarget):
                return None
            loads = _leaves(s.value)
            if any(l.attrs["mode"] != "rect" for l in loads):
                return None
            if not _ew_tree(s.value):
                return None
            sig = _ew_signature(s.value, s.target)
            if sig is None:
                return None
            groups.setdefault(sig, []).append((s, loads))
        items = []
        for s in stores:
            items.append(([_load_interval(l) for l in _leaves(s.value)], [_target_interval(s.target)]))
        if not units_independent(items):
            return None
        launches = []
        lib = R.load_library()
        for sig, members in groups.items():
            s0, _ = members[0]
            shape = s0.target.shape
            bld = EwBuilder()
            order: List[Node] = []

            def leaf(n, _order=order):
                if n.kind == "load":
                    if n not in _order:
                        _order.append(n)
                    return ("view", ("ld", _order.index(n)))
                if n.kind == "const":
                    return ("imm", (n.attrs["value"], n.dtype))
                return None
            r, dt = compile_ew(bld, s0.value, leaf)
            bld.view(("st",))
            bld.emit("ST", 0, r, dt=R.dtype_code(dt), aux=bld.view_index[("st",)])
            n_ld = len(order)
            table = np.zeros((len(members), n_ld + 1), dtype=np.int64)
            for u, (s, _) in enumerate(members):
                lds = []
                _collect_loads_in_order(s.value, lds)
                for j, l in enumerate(lds):
                    table[u, j] = l.attrs["off"]
                table[u, n_ld] = s.target.off
            contiguous = all(tuple(align_strides(l.attrs["strides"], l.shape, shape)) ==
                             dense_strides(shape) for l in order) and \
                tuple(s0.target.strides) == dense_strides(shape)

            def vf(key, _order=order, _s0=s0, _shape=shape, _n=n_ld):
                if key[0] == "ld":
                    l = _order[key[1]]
                    return mkview(self.slots[l.attrs["buf"].index], l.dtype, 0,
                                  align_strides(l.attrs["strides"], l.shape, _shape), key[1])
                t = _s0.target
                return mkview(self.slots[t.buf.index], t.dtype, 0, t.strides, _n)
            prog = program(bld, shape, len(members), n_ld + 1, vf, contiguous)
            if contiguous and self._vector_ok(prog, table):
                prog.contiguous = 2
            ut = self.dev.i64(table)

            def run(bufs, stream, status, _p=prog, _ut=ut):
                R.check(lib.ktir_ew(C.byref(_p), C.byref(bufs), C.c_void_p(_ut), stream), "ktir_ew")
            launches.append(Launch(run, "ew", meta={"prog": prog, "table": table}))
        plan = Plan("elementwise", launches, [])
        plan.info.update(units=len(stores), elems=sum(int(np.prod(s.target.shape)) for s in stores))
        return plan

    def _vector_ok(self, prog, table: np.ndarray) -> bool:
        """Whether every view of a dense program is f16, starts on a multiple of 8
        elements and stays inside its buffer in every unit (16-byte accesses, no
        zero fill or truncation needed)."""
        numel_of = {self.slots[b.index]: b.numel for b in self.trace.space.buffers}
        n = int(prog.numel)
        for i in range(prog.n_views):
            v = prog.view[i]
            if v.dtype != R.F16 or v.slot not in numel_of:
                return False
            offs = v.off + (table[:, v.unit_col] if v.unit_col >= 0 else np.zeros(1, np.int64))
            if (offs % 8).any() or (offs < 0).any() or (offs + n > numel_of[v.slot]).any():
                return False
        return True


def _collect_loads_in_order(root: Node, out: List[Node]) -> None:
    """Loads in the order compile_ew first meets them (depth-first, inputs in order)."""
    seen = set()

    def walk(n):
        if not isinstance(n, Node) or n.id in seen:
            return
        seen.add(n.id)
        if n.kind == "load":
            out.append(n)
            return
        for i in n.ins:
            walk(i)
    walk(root)


def _ew_tree(root: Node) -> bool:
    stack, seen = [root], set()
    while stack:
        n = stack.pop()
        if not isinstance(n, Node) or n.id in seen:
            continue
        seen.add(n.id)
        if n.kind == "load":
            continue
        if n.kind == "const":
            continue
        if n.kind != "ew" or n.attrs["op"] in ("bitcast",):
            return False
        stack.extend(n.ins)
    return True


def _ew_signature(root: Node, target) -> Optional[Tuple]:
    parts = []
    seen: Dict[int, int] = {}

    def walk(n):
        if isinstance(n, Const):
            parts.append(("k", repr(n.value), str(n.dtype)))
            return
        if n.id in seen:
            parts.append(("ref", seen[n.id]))
            return
        seen[n.id] = len(seen)
        if n.kind == "load":
            parts.append(("ld", n.shape, str(n.dtype), n.attrs["buf"].index,
                          tuple(n.attrs["strides"])))
            return
        if n.kind == "const":
            parts.append(("c", repr(n.attrs["value"]), str(n.dtype), n.shape))
            return
        parts.append(("ew", n.attrs.get("op"), n.attrs.get("pred"), str(n.dtype), n.shape))
        for i in n.ins:
            walk(i)
    walk(root)
    parts.append(("st", target.shape, tuple(target.strides), target.buf.index, str(target.dtype)))
    return tuple(parts)


def _elementwise_only(root: Node, leaf: Node) -> bool:
    stack, seen = [root], set()
    while stack:
        n = stack.pop()
        if not isinstance(n, Node) or n.id in seen or n is leaf:
            continue
        seen.add(n.id)
        if n.kind == "const" and not n.shape == ():
            continue
        if n.kind != "ew" or n.shape not in (root.shape, ()):
            return False
        if n.attrs["op"] in ("bitcast",):
            return False
        stack.extend(n.ins)
    return True


def _row_gather_form(iat: IATV):
    """(rows, cols, row_stride, idx_view, idx_first_elem) for table[ind(idx[s + i]), (j)]."""
    if len(iat.dims) != 2 or iat.vso is not None and not iat.vso.is_identity():
        return None
    if iat.consts:
        return None
    d0, d1 = iat.dims
    if d0["kind"] != "indirect" or d1["kind"] != "direct":
        return None
    if not isinstance(iat.vss, BoxSet) or iat.vss.lo != (0, 0):
        return None
    R_, C_ = iat.vss.hi
    if (R_, C_) != tuple(iat.shape):
        return None
    par = iat.parent
    if len(par.strides) != 2 or par.strides[1] != 1:
        return None
    # the direct subscript must be exactly the column variable
    lin = linearize(_subst(d1["expr"], iat.refs), 2)
    if lin is None or lin[0] != [0, 1] or lin[2] != 0:
        return None
    if len(d0["exprs"]) != 1:
        return None
    view = iat.views[d0["view"]]
    if len(view.strides) != 1:
        return None
    lin = linearize(_subst(d0["exprs"][0], iat.refs), 2)
    if lin is None or lin[0] != [1, 0]:
        return None
    first = lin[2] * view.strides[0]
    if view.strides[0] != 1:
        return None
    return (int(R_), int(C_), int(par.strides[0]), view, int(first))


def _subst(e, refs):
    from .affine import substitute_refs
    return substitute_refs(e, lambda leaf: ("c", int(refs[leaf[1]])))


def _resolve_buffer(trace: Trace, view) -> Optional[Any]:
    return trace.space.find(view.byte_address)


def _softmax_form(v: Node):
    """Match out = f16(exp(x - max(x)) / sum(exp(x - max(x)))) with x = [ext](load)."""
    def strip_cast(n):
        return n.ins[0] if isinstance(n, Node) and n.kind == "ew" and n.attrs["op"] == "cast" else n

    def bc_of_reduce(n, comb):
        # broadcast (via generic indexing map or splat/extract) of a row reduction
        if not isinstance(n, Node):
            return None
        if n.kind == "bcast" and n.attrs["map"] == (0,):
            r = n.ins[0]
            if r.kind == "reduce" and r.attrs["dim"] == 1 and r.attrs["combiner"] == comb:
                return r.ins[0]
        return None

    root = v
    if not (isinstance(root, Node) and root.dtype == np.float16):
        return None
    body = strip_cast(root) if root.kind == "ew" and root.attrs["op"] == "cast" else root
    if body.kind != "ew" or body.attrs["op"] != "div":
        return None
    e, den = body.ins
    if isinstance(e, Node) and e.kind == "bcast":
        e = e.ins[0] if e.attrs["map"] == (0, 1) else e
    src = bc_of_reduce(den, "arith.addf")
    if src is None:
        return None
    if src is not e and not (src.kind == "bcast" and src.ins[0] is e):
        if not (isinstance(src, Node) and src.kind == "bcast" and src.attrs["map"] == (0, 1)
                and src.ins[0] is e):
            return None
    if e.kind != "ew" or e.attrs["op"] != "exp":
        return None
    d = e.ins[0]
    if d.kind != "ew" or d.attrs["op"] != "sub":
        return None
    x, mx = d.ins
    if isinstance(x, Node) and x.kind == "bcast" and x.attrs["map"] == (0, 1):
        x = x.ins[0]
    xs = bc_of_reduce(mx, "arith.maxnumf")
    if xs is None:
        return None
    if xs is not x:
        return None
    ld = strip_cast(x)
    if not (isinstance(ld, Node) and ld.kind == "load" and ld.attrs["mode"] == "rect"):
        return None
    cf16 = e.dtype == np.float16
    if not cf16 and not (x.kind == "ew" and x.attrs["op"] == "cast" and x.dtype == np.float32):
        return None
    return ld, cf16


# ---------------------------------------------------------------------------
# generic executor
# ---------------------------------------------------------------------------

class _Val:
    """Where a node's value lives: an arena/buffer view, or an immediate."""
    __slots__ = ("slot", "off", "strides", "dtype", "imm", "dense")

    def __init__(self, slot=None, off=0, strides=(), dtype=None, imm=None, dense=False):
        self.slot = slot
        self.off = off
        self.strides = tuple(strides)
        self.dtype = np.dtype(dtype) if dtype is not None else None
        self.imm = imm
        self.dense = dense


class GenericExecutor:
    """Core-by-core, node-by-node execution in program order."""

    def __init__(self, low: Lowerer):
        self.low = low
        self.trace = low.trace
        self.lib = R.load_library()
        self.launches: List[Launch] = []
        self.arena_bytes = 0
        self.vals: Dict[int, _Val] = {}
        self.dense_uploads: List[Tuple[int, np.ndarray]] = []

    def alloc(self, nbytes: int, itemsize: int) -> int:
        off = (self.arena_bytes + 255) & ~255
        self.arena_bytes = off + max(int(nbytes), 1)
        return off // itemsize

    def build(self) -> Plan:
        tr = self.trace
        # the trace lists nodes and stores in the order the call executes them
        # (core after core, and across a collective every core's part before
        # it, then every core's part after it); replay that order, a store
        # preceding every node created after it
        needed = self._needed(tr.stores)
        nodes = [n for n in tr.nodes if n.id in needed]
        stores = sorted(tr.stores, key=lambda s: (self._created_before(s), s.seq))
        order: List[Any] = []
        si = 0
        for n in nodes:
            while si < len(stores) and self._created_before(stores[si]) <= n.id:
                order.append(stores[si])
                si += 1
            order.append(n)
        order.extend(stores[si:])
        for item in order:
            if isinstance(item, Node):
                self.node(item)
            else:
                self.store(item)
        plan = Plan("generic", self.launches, [], arena_bytes=self.arena_bytes, status_check=True)
        plan.info["dense_uploads"] = self.dense_uploads
        return plan

    @staticmethod
    def _created_before(s: Store) -> int:
        return s.mark

    def _needed(self, stores: List[Store]) -> set:
        need, stack = set(), [s.value for s in stores]
        while stack:
            n = stack.pop()
            if not isinstance(n, Node) or n.id in need:
                continue
            need.add(n.id)
            stack.extend(n.ins)
            if n.kind == "load" and n.attrs["mode"] == "indirect":
                pass
        return need

    # -- views ------------------------------------------------------------------------
    def arena_dense(self, n: Node) -> _Val:
        off = self.alloc(n.nbytes, n.dtype.itemsize)
        return _Val(R.ARENA_SLOT, off, dense_strides(n.shape), n.dtype, dense=True)

    def view_of(self, n: Node) -> _Val:
        v = self.vals.get(n.id)
        if v is None:
            raise RuntimeError(f"value of {n} not materialised")
        return v

    def materialize(self, n: Node) -> _Val:
        """Dense arena copy of node n (which has a value already)."""
        v = self.view_of(n)
        if v.imm is None and v.slot == R.ARENA_SLOT and v.dense:
            return v
        out = self.arena_dense(n)
        self._ew_copy(n, v, out)
        return out

    def _ew_copy(self, n: Node, src: _Val, dst: _Val, dst_dtype=None) -> None:
        shape = n.shape if n.shape else (1,)
        b = EwBuilder()
        if src.imm is not None:
            r = b.imm(src.imm, n.dtype)
        else:
            r = b.alloc()
            b.emit("LD", r, aux=b.view("src"))
        b.view("dst")
        b.emit("ST", 0, r, dt=R.dtype_code(n.dtype), aux=b.view_index["dst"])

        def vf(key):
            if key == "src":
                st = src.strides if n.shape else (0,)
                return mkview(src.slot, src.dtype, src.off, st)
            st = dst.strides if n.shape else (0,)
            return mkview(dst.slot, dst_dtype if dst_dtype is not None else dst.dtype, dst.off, st)
        self._launch_ew(program(b, shape, 1, 0, vf))

    def _offsets(self, dense: _Val, tile: _Val, positions: np.ndarray, scatter: bool) -> None:
        """Gather tile[positions] into dense, or scatter dense into
        tile[positions]; both are dense arena values."""
        if positions.size == 0:
            return
        optr = self.low.dev.i64(positions)
        d = R.KtirOffsetsDesc()
        d.buf = mkview(R.ARENA_SLOT, tile.dtype, tile.off, ())
        d.dense = mkview(R.ARENA_SLOT, dense.dtype, dense.off, ())
        d.count = positions.size
        d.n_units = 1
        d.scatter = 1 if scatter else 0
        lib = self.lib

        def run(bufs, stream, status, _d=d, _o=optr):
            R.check(lib.ktir_offsets(C.byref(_d), C.byref(bufs), None, C.c_void_p(_o), stream),
                    "ktir_offsets")
        self.launches.append(Launch(run, "scatter" if scatter else "gather"))

    def _launch_ew(self, prog) -> None:
        lib = self.lib

        def run(bufs, stream, status, _p=prog):
            R.check(lib.ktir_ew(C.byref(_p), C.byref(bufs), None, stream), "ktir_ew")
        self.launches.append(Launch(run, "ew"))

    # -- nodes --------------------------------------------------------------------------
    def node(self, n: Node) -> None:
        k = n.kind
        if k == "const":
            self.vals[n.id] = _Val(imm=n.attrs["value"], dtype=n.dtype)
        elif k == "dense":
            out = self.arena_dense(n)
            self.dense_uploads.append((out.off * n.dtype.itemsize,
                                       np.ascontiguousarray(n.attrs["value"], dtype=n.dtype)))
            self.vals[n.id] = out
        elif k == "load":
            self.load(n)
        elif k == "ew":
            self.ew(n)
        elif k == "iota":
            out = self.arena_dense(n)
            b = EwBuilder()
            r = b.alloc()
            b.emit("IOTA", r, aux=n.attrs["dim"], dt=R.I64)
            b.view("dst")
            b.emit("ST", 0, r, dt=R.I64, aux=0)
            self._launch_ew(program(b, n.shape, 1, 0,
                                    lambda key: mkview(R.ARENA_SLOT, n.dtype, out.off, out.strides)))
            self.vals[n.id] = out
        elif k in ("bcast", "transpose", "reshape", "splat", "extract", "slice"):
            self.view_node(n)
        elif k == "assemble":
            # zero tile with each piece copied in at its offset (distributed load);
            # a piece of scattered points is placed element by element
            out = self.arena_dense(n)
            self._ew_copy(n, _Val(imm=n.dtype.type(0), dtype=n.dtype), out)
            for piece, at in zip(n.ins, n.attrs["at"]):
                if isinstance(at, np.ndarray):
                    self._offsets(self.materialize(piece), out, at, scatter=True)
                    continue
                off = out.off + sum(a * st for a, st in zip(at, out.strides))
                self._ew_copy(piece, self.view_of(piece), _Val(R.ARENA_SLOT, off, out.strides,
                                                               n.dtype))
            self.vals[n.id] = out
        elif k == "pick":
            # the elements at row-major positions of a tile, in order
            out = self.arena_dense(n)
            src = self.materialize(n.ins[0])
            self._offsets(out, src, n.attrs["positions"], scatter=False)
            self.vals[n.id] = out
        elif k == "reduce":
            self.reduce(n)
        elif k == "matmul":
            self.matmul(n)
        else:
            raise NotImplementedError(f"generic executor: node kind {k}")

    def view_node(self, n: Node) -> None:
        src = n.ins[0]
        sv = self.view_of(src)
        k = n.kind
        if sv.imm is not None and k != "extract":
            self.vals[n.id] = _Val(imm=sv.imm, dtype=n.dtype)
            return
        if k == "slice":
            if sv.imm is not None:
                self.vals[n.id] = _Val(imm=sv.imm, dtype=n.dtype)
                return
            off = sv.off + sum(a * st for a, st in zip(n.attrs["at"], sv.strides))
            self.vals[n.id] = _Val(sv.slot, off, sv.strides, sv.dtype)
            return
        if k == "extract":
            if sv.imm is not None:
                self.vals[n.id] = _Val(imm=sv.imm, dtype=n.dtype)
                return
            off = sv.off + sum(i * s for i, s in zip(n.attrs["index"], sv.strides))
            self.vals[n.id] = _Val(sv.slot, off, (), sv.dtype)
        elif k == "splat":
            self.vals[n.id] = _Val(sv.slot, sv.off, (0,) * len(n.shape), sv.dtype)
        elif k == "transpose":
            perm = n.attrs["perm"]
            self.vals[n.id] = _Val(sv.slot, sv.off, tuple(sv.strides[i] for i in perm), sv.dtype)
        elif k == "bcast":
            m = n.attrs["map"]
            st = [0] * len(n.shape)
            for i, d in enumerate(m):
                st[d] = 0 if (src.shape[i] == 1 and n.shape[d] != 1) else sv.strides[i]
            self.vals[n.id] = _Val(sv.slot, sv.off, tuple(st), sv.dtype)
        elif k == "reshape":
            if not sv.dense:
                sv = self.materialize(src)
            self.vals[n.id] = _Val(sv.slot, sv.off, dense_strides(n.shape), sv.dtype, dense=True)

    def load(self, n: Node) -> None:
        a = n.attrs
        out = self.arena_dense(n)
        slot = self.low.slots[a["buf"].index]
        if a["mode"] == "rect":
            self._ew_copy(n, _Val(slot, a["off"], a["strides"], n.dtype), out)
        elif a["mode"] == "coords":
            offs = self.low.dev.i64(a["offsets"])
            d = R.KtirOffsetsDesc()
            d.buf = mkview(slot, n.dtype, a["off"], ())
            d.dense = mkview(R.ARENA_SLOT, n.dtype, out.off, ())
            d.count = a["offsets"].size
            d.n_units = 1
            d.scatter = 0
            lib = self.lib

            def run(bufs, stream, status, _d=d, _o=offs):
                R.check(lib.ktir_offsets(C.byref(_d), C.byref(bufs), None, C.c_void_p(_o), stream),
                        "ktir_offsets")
            self.launches.append(Launch(run, "gather"))
        else:
            self._indirect(n.attrs["iat"], out, n.dtype, scatter=False)
        self.vals[n.id] = out

    def _indirect(self, iat: IATV, dense: _Val, dtype, scatter: bool) -> None:
        direct, idx_offs, ind_views, strides = indirect_tables(iat)
        pbuf = self.trace.space.find(iat.parent.byte_address)
        d = R.KtirIndirectDesc()
        d.buf = mkview(self.low.slots[pbuf.index], np.dtype(dtype),
                       (iat.parent.byte_address - pbuf.byte_base) // np.dtype(dtype).itemsize, ())
        d.dense = mkview(R.ARENA_SLOT, np.dtype(dtype), dense.off, ())
        d.count = direct.size
        d.n_units = 1
        d.n_ind = len(ind_views)
        d.scatter = 1 if scatter else 0
        for k, (v, s) in enumerate(zip(ind_views, strides)):
            ib = self.trace.space.find(v.byte_address)
            if ib is None:
                raise ValueError(f"Read from unmapped address 0x{v.byte_address:x}")
            d.idx_slot[k] = self.low.slots[ib.index]
            d.idx_dtype[k] = R.dtype_code(ib.dtype)
            d.stride[k] = s
            base = (v.byte_address - ib.byte_base) // ib.dtype.itemsize
            idx_offs[k] = idx_offs[k] + base
        dptr = self.low.dev.i64(direct)
        iptr = self.low.dev.i64(np.concatenate(idx_offs) if idx_offs else np.zeros(1, np.int64))
        lib = self.lib

        def run(bufs, stream, status, _d=d, _dp=dptr, _ip=iptr):
            R.check(lib.ktir_indirect(C.byref(_d), C.byref(bufs), None, C.c_void_p(_dp),
                                      C.c_void_p(_ip), C.c_void_p(status), stream), "ktir_indirect")
        self.launches.append(Launch(run, "indirect"))

    def ew(self, n: Node) -> None:
        out = self.arena_dense(n)
        shape = n.shape if n.shape else (1,)
        b = EwBuilder()
        keys: Dict[Any, _Val] = {}

        def leaf(x):
            if x is n:
                return None
            v = self.vals.get(x.id)
            if v is None:
                return None
            if v.imm is not None:
                return ("imm", (v.imm, x.dtype))
            key = ("v", x.id)
            keys[key] = (v, x)
            return ("view", key)
        r, dt = compile_ew(b, n, leaf)
        b.view("dst")
        b.emit("ST", 0, r, dt=R.dtype_code(dt), aux=b.view_index["dst"])

        def vf(key):
            if key == "dst":
                return mkview(R.ARENA_SLOT, n.dtype, out.off, out.strides if n.shape else (0,))
            v, x = keys[key]
            st = align_strides(v.strides, x.shape, n.shape) if n.shape else (0,)
            if not x.shape:
                st = (0,) * len(shape)
            return mkview(v.slot, v.dtype, v.off, st)
        self._launch_ew(program(b, shape, 1, 0, vf))
        self.vals[n.id] = out

    def reduce(self, n: Node) -> None:
        src = n.ins[0]
        comb = n.attrs["combiner"]
        if isinstance(comb, tuple):
            if comb[0] == "swapped":
                comb = comb[1]
            else:
                raise NotImplementedError("linalg.reduce with a multi-op combiner region")
        if comb not in COMBINER:
            raise NotImplementedError(f"linalg.reduce combiner {comb}")
        opname = COMBINER[comb]
        if is_float(n.dtype) != opname.startswith("F"):
            if is_float(n.dtype):
                raise NotImplementedError(f"{comb} on float tiles")
            opname = {"FADD": "IADD", "FMUL": "IMUL", "FMAXNUM": "IMAX", "FMINNUM": "IMIN",
                      "FMAXIMUM": "IMAX", "FMINIMUM": "IMIN"}.get(opname, opname)
        sv = self.materialize(src) if self.view_of(src).imm is None else self.materialize(src)
        dim = n.attrs["dim"]
        shp = src.shape
        outer = int(np.prod(shp[:dim])) if dim > 0 else 1
        inner = int(np.prod(shp[dim + 1:])) if dim + 1 < len(shp) else 1
        out = self.arena_dense(n)
        tmp = self.alloc(src.nbytes, src.dtype.itemsize)
        d = R.KtirReduceDesc()
        d.combiner = OP[opname]
        d.dt = R.dtype_code(n.dtype)
        d.n_units = 1
        d.outer, d.n, d.inner = outer, shp[dim], inner
        d.in_off, d.out_off, d.tmp_off = sv.off, out.off, tmp
        d.unit_stride = 0
        d.in_slot = d.out_slot = R.ARENA_SLOT
        lib = self.lib

        def run(bufs, stream, status, _d=d):
            R.check(lib.ktir_reduce(C.byref(_d), C.byref(bufs), stream), "ktir_reduce")
        self.launches.append(Launch(run, "reduce"))
        self.vals[n.id] = out

    def _dense_aligned(self, n: Node) -> _Val:
        """Row-major arena copy of n starting on a 16-byte boundary (n's own
        value when it already is one)."""
        v = self.view_of(n)
        if (v.imm is None and v.slot == R.ARENA_SLOT and v.dense
                and (v.off * n.dtype.itemsize) % 16 == 0):
            return v
        out = self.arena_dense(n)     # arena allocations start on 256-byte boundaries
        self._ew_copy(n, v, out)
        return out

    def _matmul_tc(self, n: Node, a: Node, bnode: Node) -> bool:
        """An f16 x f16 -> f16 product on the tensor cores
        (ktir_gemm_f16_blocked with one block of all of K: an f32 sum rounded
        to f16 once, as NumPy's half matmul); False when the operands do not
        fit its TMA tiles (row strides must be multiples of 16 bytes)."""
        f16 = np.dtype(np.float16)
        if not (a.dtype == bnode.dtype == n.dtype == f16) or len(a.shape) != 2 \
                or len(bnode.shape) != 2 or len(n.shape) != 2:
            return False
        m, k = a.shape
        nn = bnode.shape[1]
        if m < 1 or k < 1 or nn < 1 or k % 8 or nn % 8 or -(-nn // 128) > 65535:
            return False
        va, vb = self._dense_aligned(a), self._dense_aligned(bnode)
        out = self.arena_dense(n)
        d = R.KtirGemmBlockedDesc()
        d.lda, d.ldb, d.ldc = k, nn, nn
        d.m, d.n, d.k = m, nn, k
        d.block_k, d.acc_f16 = 0, 0
        lib = self.lib
        offs = (va.off * 2, vb.off * 2, out.off * 2)

        def run(bufs, stream, status, _d=d, _o=offs):
            arena = bufs.base[R.ARENA_SLOT]
            _d.a, _d.b, _d.c = arena + _o[0], arena + _o[1], arena + _o[2]
            _d.status = status
            R.check(lib.ktir_gemm_f16_blocked(C.byref(_d), stream), "ktir_gemm_f16_blocked")
        self.launches.append(Launch(run, "matmul_tc"))
        self.vals[n.id] = out
        return True

    def matmul(self, n: Node) -> None:
        a, bnode = n.ins
        if self._matmul_tc(n, a, bnode):
            return
        va, vb = self.view_of(a), self.view_of(bnode)
        if va.imm is not None:
            va = self.materialize(a)
        if vb.imm is not None:
            vb = self.materialize(bnode)
        out = self.arena_dense(n)
        if len(n.shape) != 2 or len(a.shape) != 2:
            raise NotImplementedError("generic matmul handles 2-D tiles")
        d = R.KtirMatmulDesc()
        d.batch, d.m, d.n, d.k = 1, a.shape[0], bnode.shape[1], a.shape[1]
        d.a = mkview(va.slot, va.dtype, va.off, (0,) + tuple(va.strides))
        d.b = mkview(vb.slot, vb.dtype, vb.off, (0,) + tuple(vb.strides))
        d.out = mkview(R.ARENA_SLOT, n.dtype, out.off, (0,) + tuple(out.strides))
        d.n_units, d.unit_cols = 1, 0
        lib = self.lib

        def run(bufs, stream, status, _d=d):
            R.check(lib.ktir_matmul(C.byref(_d), C.byref(bufs), None, stream), "ktir_matmul")
        self.launches.append(Launch(run, "matmul"))
        self.vals[n.id] = out

    # -- stores -----------------------------------------------------------------------------
    def store(self, s: Store) -> None:
        v = s.value
        sv = self.view_of(v)
        t = s.target
        if isinstance(t, RectTarget):
            slot = self.low.slots[t.buf.index]
            # the value's elements in C order land on the box in C order
            if sv.imm is None and not sv.dense and tuple(v.shape) != tuple(t.shape):
                sv = self.materialize(v)
            src = sv if tuple(v.shape) == tuple(t.shape) else _Val(
                sv.slot, sv.off, dense_strides(t.shape), sv.dtype, sv.imm, True)
            if sv.imm is not None:
                src = sv
            node = Node(-1, "store", t.shape, v.dtype)
            self._ew_copy(node, src, _Val(slot, t.off, t.strides, t.dtype), t.dtype)
        elif isinstance(t, CoordTarget):
            dv = self.materialize(v) if sv.imm is None else self._fill(v)
            offs = t.offsets.copy()
            # keep only the last writer of each duplicated offset
            _, last = np.unique(offs[::-1], return_index=True)
            keep = np.zeros(offs.size, bool)
            keep[offs.size - 1 - last] = True
            offs[~keep] = -1
            optr = self.low.dev.i64(offs)
            d = R.KtirOffsetsDesc()
            d.buf = mkview(self.low.slots[t.buf.index], t.dtype, t.off, ())
            d.dense = mkview(R.ARENA_SLOT, v.dtype, dv.off, ())
            d.count = offs.size
            d.n_units = 1
            d.scatter = 1
            lib = self.lib

            def run(bufs, stream, status, _d=d, _o=optr):
                R.check(lib.ktir_offsets(C.byref(_d), C.byref(bufs), None, C.c_void_p(_o), stream),
                        "ktir_offsets")
            self.launches.append(Launch(run, "scatter"))
        else:
            dv = self.materialize(v) if sv.imm is None else self._fill(v)
            self._indirect(t.iat, dv, v.dtype, scatter=True)

    def _fill(self, v: Node) -> _Val:
        out = self.arena_dense(v)
        self._ew_copy(v, self.view_of(v), out)
        return out


def indirect_tables(iat: IATV):
    """Per-point direct element offsets and index-tensor element offsets.

    Enumerates the variable space exactly as the reference does (row-major
    box, or sorted by a permutation variables_space_order —
    ktir_cpu/ops/memory_ops.py:170-186) and evaluates the subscripts
    vectorised.  Returns (direct[npts], [idx_off_k[npts]], [view_k], [stride_k])
    with offsets relative to the parent / index view base.
    """
    from .affine import eval_expr
    pts = iat.vss.enumerate_array(iat.shape)
    if iat.vso is not None and len(pts):
        keys = np.stack([np.broadcast_to(np.asarray(k, np.int64), (pts.shape[0],))
                         for k in iat.vso.eval(list(pts.T))], axis=1)
        pts = pts[np.lexsort(keys.T[::-1])]
    n = pts.shape[0]
    cols = [pts[:, i].astype(np.int64) for i in range(pts.shape[1])]
    for i, v in iat.consts.items():
        cols[i] = np.full(n, v, np.int64)

    def ev(e):
        return np.broadcast_to(np.asarray(eval_expr(e, cols, (), iat.refs), np.int64), (n,))
    direct = np.zeros(n, np.int64)
    idx_offs, views, strides = [], [], []
    pstr = iat.parent.strides
    for k, d in enumerate(iat.dims):
        if d["kind"] == "direct":
            direct = direct + ev(d["expr"]) * pstr[k]
        else:
            view = iat.views[d["view"]]
            off = np.zeros(n, np.int64)
            for e, s in zip(d["exprs"], view.strides):
                off = off + ev(e) * s
            idx_offs.append(off)
            views.append(view)
            strides.append(pstr[k])
    return direct, idx_offs, views, strides
