"""Host shadow pass: per-core scalar execution that records tile work as a DAG.

This replaces the reference's execution engine (ktir_cpu/grid.py:471-570
running every op through the handler registry, dialects/registry.py:87-115)
for one purpose: it evaluates everything that is *scalar* on the host —
core ids, loop bounds, index arithmetic, memory views and access tiles,
exactly as the reference does — and records everything that touches *tile
data* as nodes of a dataflow graph.  Tile data never exists on the host; the
graph is lowered onto device kernels by :mod:`ktir_cpu_b200.lower`.

What is replicated here because results depend on it:

* core order and grid coordinates (grid.py:402-416, x fastest);
* the HBM address space: stick-aligned allocations from 0x10000, access
  resolution to the allocation holding the start address, zero fill past its
  end on reads and truncation on writes (memory.py:97-288) — recorded as the
  bounds every device access is clamped to;
* LX accounting with scoped frees and the exact MemoryError text
  (grid.py:204-311, interpreter.py:216-226, control_ops.py:77-167);
* NumPy dtype promotion for every tile op, including the float16 coercion of
  scalar operands in float binops (dialects/_helpers.py:35-54) and the
  float32 evaluation of math ops (ops/math_ops.py:30-268);
* the error conventions of the reference (ValueError for unknown ops and
  unmapped reads, IndexError for negative indices — raised after the device
  run reports them — MemoryError for LX overflow).

Data-dependent control flow or addressing (a scalar extracted from a tile
steering scf.for / scf.if or an access tile) is rejected with
NotImplementedError: every supported program has a data-independent schedule.
"""

from __future__ import annotations

import bisect
import operator
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np

from .affine import AffineMap, BoxSet
from .ir import IRFunction, Operation, iter_ops, linalg_block_args

STICK = 128
LX_CAPACITY = 2 * 1024 * 1024
# LX scratchpads live in the trace's address space apart from HBM: core c's
# byte b is at LX_BASE + c * LX_SPAN + b
LX_BASE = 1 << 50
LX_SPAN = 1 << 36


def lx_address(core: int, byte: int) -> int:
    return LX_BASE + core * LX_SPAN + byte

NP = {
    "f16": np.float16, "fp16": np.float16, "float16": np.float16,
    "f32": np.float32, "float32": np.float32,
    "i1": np.bool_, "i32": np.int32, "si32": np.int32, "index": np.int32,
    "i64": np.int64, "si64": np.int64,
}
LABEL = {np.dtype(np.float16): "f16", np.dtype(np.float32): "f32", np.dtype(np.int32): "i32",
         np.dtype(np.int64): "i64", np.dtype(np.bool_): "i1", np.dtype(np.uint32): "ui32"}


def np_dtype(name: str) -> np.dtype:
    if name in ("fp8", "mxfp8"):
        raise NotImplementedError(f"dtype {name!r} is a placeholder")
    try:
        return np.dtype(NP[name])
    except KeyError:
        raise ValueError(f"Unsupported KTIR dtype: {name!r}")


def bpe(name: str) -> int:
    return np_dtype(name).itemsize


# ---------------------------------------------------------------------------
# host-side model of the simulated HBM address space
# ---------------------------------------------------------------------------

@dataclass
class Buffer:
    index: int
    name: str
    byte_base: int
    nbytes: int
    dtype: np.dtype
    shape: Tuple[int, ...]

    @property
    def numel(self) -> int:
        return self.nbytes // self.dtype.itemsize


class AddressSpace:
    def __init__(self) -> None:
        self.buffers: List[Buffer] = []
        self._starts: List[int] = []
        self.next_ptr = 0x10000

    def allocate(self, name: str, nbytes: int, dtype, shape) -> int:
        ptr = self.next_ptr
        self.next_ptr = (ptr + nbytes + STICK - 1) & ~(STICK - 1)
        buf = Buffer(len(self.buffers), name, ptr, nbytes, np.dtype(dtype), tuple(shape))
        self.buffers.append(buf)
        k = bisect.bisect_right(self._starts, ptr)
        self._starts.insert(k, ptr)
        return ptr // STICK

    def add_fixed(self, name: str, byte_addr: int, nbytes: int, dtype, shape) -> Buffer:
        buf = Buffer(len(self.buffers), name, byte_addr, nbytes, np.dtype(dtype), tuple(shape))
        self.buffers.append(buf)
        k = bisect.bisect_right(self._starts, byte_addr)
        self._starts.insert(k, byte_addr)
        return buf

    def find(self, addr: int) -> Optional[Buffer]:
        by_start = {b.byte_base: b for b in self.buffers}
        if addr in by_start:
            return by_start[addr]
        k = bisect.bisect_right(self._starts, addr) - 1
        if k >= 0:
            b = by_start[self._starts[k]]
            if b.byte_base < addr < b.byte_base + b.nbytes:
                return b
        return None


# ---------------------------------------------------------------------------
# graph
# ---------------------------------------------------------------------------

class Node:
    __slots__ = ("id", "kind", "shape", "dtype", "ins", "attrs", "label", "pyscalar", "core")

    def __init__(self, id, kind, shape, dtype, ins=(), attrs=None, label=None, pyscalar=False,
                 core=0):
        self.id = id
        self.kind = kind
        self.shape = tuple(int(s) for s in shape)
        self.dtype = np.dtype(dtype)
        self.ins = tuple(ins)
        self.attrs = attrs or {}
        self.label = label or LABEL.get(self.dtype, "f16")
        self.pyscalar = pyscalar
        self.core = core

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def nbytes(self) -> int:
        return self.numel * self.dtype.itemsize

    def proto(self):
        """A NumPy value with this node's dtype behaviour, for promotion queries."""
        if self.shape:
            return np.zeros((1,) * len(self.shape), dtype=self.dtype)
        if self.pyscalar:
            return 0.0 if self.dtype.kind == "f" else (False if self.dtype.kind == "b" else 0)
        return self.dtype.type(0)

    def __repr__(self):
        return f"<{self.kind}#{self.id} {self.shape} {self.dtype}>"


@dataclass
class Const:
    """Immediate scalar operand of an elementwise op (already in its final dtype)."""
    value: Any
    dtype: np.dtype


@dataclass
class RectTarget:
    buf: Buffer
    off: int                    # element offset of the tile origin inside the buffer
    shape: Tuple[int, ...]
    strides: Tuple[int, ...]
    dtype: np.dtype


@dataclass
class CoordTarget:
    buf: Buffer
    off: int
    offsets: np.ndarray         # element offsets relative to off, enumeration order
    shape: Tuple[int, ...]      # tile shape the values come in
    dtype: np.dtype


@dataclass
class IndirectTarget:
    iat: "IATV"


@dataclass
class Store:
    core: int
    seq: int
    value: Node
    target: Any
    mark: int = 0               # number of graph nodes created before this store


# ---------------------------------------------------------------------------
# tracer values
# ---------------------------------------------------------------------------

@dataclass
class MemRefV:
    stick: int                  # HBM: stick index; LX: byte address in its scratchpad
    shape: Tuple[int, ...]
    strides: List[int]
    space: str
    dtype: str
    cset: Any = None
    lx_core: Optional[int] = None

    @property
    def byte_address(self) -> int:
        if self.space == "LX":
            return lx_address(self.lx_core, self.stick)
        return self.stick * STICK


@dataclass
class DistMemRefV:
    """ktdp.construct_distributed_memory_view: partitions in global coordinates."""
    parts: List[MemRefV]
    shape: Tuple[int, ...]
    dtype: str


@dataclass
class DistAccessV:
    """An access tile over a distributed view, resolved to the partitions it
    touches: (partition, covered box in global coordinates, partition origin)."""
    base: Tuple[int, ...]
    shape: Tuple[int, ...]
    dtype: str
    pieces: List[Tuple[MemRefV, Any, Tuple[int, ...]]]


@dataclass
class AccessTileV:
    byte: int
    shape: Tuple[int, ...]
    strides: List[int]
    dtype: str
    cset: Any
    order: Optional[AffineMap]


@dataclass
class IATV:
    parent: MemRefV
    shape: Tuple[int, ...]
    dims: List[dict]            # kind: direct(expr) / indirect(view, exprs); refs resolved
    views: List[MemRefV]
    vss: Any
    vso: Optional[AffineMap]
    consts: Dict[int, int]      # intermediate variable index -> outer SSA scalar value
    refs: Dict[str, int]

    def signature(self):
        return (id(self.vss), self.vso.source if self.vso else None, tuple(self.consts.items()),
                tuple(sorted(self.refs.items())))


@dataclass
class FutureV:
    """A core's ktdp.tile_future: its partial and the sets naming its group."""
    partial: Any
    producer_set: Any
    groups_set: Any
    group: int


class _Yield:
    __slots__ = ("values",)

    def __init__(self, values):
        self.values = values


def _is_scalar(v) -> bool:
    return isinstance(v, (int, float, bool, np.integer, np.floating, np.bool_)) or \
        (isinstance(v, Node) and not v.shape)


def _is_tile(v) -> bool:
    return isinstance(v, Node) and bool(v.shape)


def _elements(res, operands) -> int:
    """Element count an op is charged for: its tile result, else its first
    tile operand, else 1 (ktir_cpu/latency.py:340-347)."""
    if isinstance(res, Node) and not res.pyscalar:
        return int(np.prod(res.shape)) if res.shape else 1
    for v in operands:
        if isinstance(v, Node) and not v.pyscalar:
            return int(np.prod(v.shape)) if v.shape else 1
    return 1


def _concrete(v) -> bool:
    return isinstance(v, (int, float, bool, np.integer, np.floating, np.bool_))


class DataDependentError(NotImplementedError):
    pass


def _need_int(v, what: str) -> int:
    if isinstance(v, Node):
        raise DataDependentError(
            f"{what} depends on tile data; this backend needs a data-independent schedule")
    return int(v)


# ---------------------------------------------------------------------------
# the tracer
# ---------------------------------------------------------------------------

class CoreState:
    def __init__(self, cid: int, pos: Tuple[int, int, int]):
        self.core_id = cid
        self.pos = pos
        self.scopes: List[Dict[str, Any]] = [{}]
        self.lx_used = 0
        self.lx_bytes: Dict[str, int] = {}

    def push(self):
        self.scopes.append({})

    def pop(self):
        scope = self.scopes.pop()
        for n in scope:
            self.untrack(n)

    def set(self, n, v):
        self.scopes[-1][n] = v

    def get(self, n):
        for s in reversed(self.scopes):
            if n in s:
                return s[n]
        raise KeyError(f"Value '{n}' not found in core {self.core_id}")

    def has(self, n) -> bool:
        return any(n in s for s in self.scopes)

    def track(self, n, size):
        if self.lx_used + size > LX_CAPACITY:
            raise MemoryError(
                f"LX scratchpad overflow on core {self.core_id}: requested {size} bytes, "
                f"available {LX_CAPACITY - self.lx_used} bytes (capacity {LX_CAPACITY} bytes)")
        self.lx_bytes[n] = size
        self.lx_used += size

    def untrack(self, n):
        if n in self.lx_bytes:
            self.lx_used -= self.lx_bytes.pop(n)


class Trace:
    """Result of tracing one function call: graph nodes + ordered stores."""

    def __init__(self, space: AddressSpace, grid):
        self.space = space
        self.grid = grid
        self.nodes: List[Node] = []
        self.stores: List[Store] = []
        self.lx_peak: Dict[int, int] = {}


class Tracer:
    def __init__(self, func: IRFunction, space: AddressSpace, scalars: Dict[str, Any],
                 pointers: Dict[str, int], rewrites: Optional[Dict[int, Any]] = None,
                 latency=None):
        self.func = func
        self.space = space
        self.scalars = scalars
        self.pointers = pointers
        self.trace = Trace(space, func.grid)
        self.core: Optional[CoreState] = None
        self.seq = 0
        self.rewrites = rewrites or {}
        # LatencyTape receiving one record per executed op (optional)
        self.lat = latency

    # -- node helpers ----------------------------------------------------------
    def node(self, kind, shape, dtype, ins=(), attrs=None, label=None, pyscalar=False) -> Node:
        n = Node(len(self.trace.nodes), kind, shape, dtype, ins, attrs, label, pyscalar,
                 self.core.core_id if self.core else 0)
        self.trace.nodes.append(n)
        return n

    def const_tile(self, value, shape, dtype, label=None) -> Node:
        return self.node("const", shape, dtype, (), {"value": value}, label)

    # -- driver ----------------------------------------------------------------
    def run(self) -> Trace:
        nx, ny, nz = self.func.grid
        n = nx * ny * nz
        states = []
        for cid in range(n):
            z, r = divmod(cid, nx * ny)
            y, x = divmod(r, nx)
            st = CoreState(cid, (x, y, z))
            for aname, _ in self.func.arguments:
                key = aname.lstrip("%")
                if key in self.pointers:
                    st.set(aname, self.pointers[key])
                elif key in self.scalars:
                    st.set(aname, self.scalars[key])
            states.append(st)
        # Cores run one after another.  A ktdp.inter_tile_reduce is a
        # collective over the whole grid: every core runs up to it, then the
        # ring result of every consumer is formed, then every core runs on to
        # the next one (the reference's scheduler observes the same order:
        # no core passes the ring before all cores reached it).
        segments: List[List[Operation]] = [[]]
        collectives: List[Operation] = []
        for op in self.func.operations:
            if op.op_type == "ktdp.inter_tile_reduce":
                collectives.append(op)
                segments.append([])
            else:
                for o in iter_ops([op]):
                    if o.op_type == "ktdp.inter_tile_reduce":
                        raise NotImplementedError(
                            "ktdp.inter_tile_reduce inside a region is not supported by the "
                            "B200 backend (only at the top level of the function)")
                segments[-1].append(op)
        for si, seg in enumerate(segments):
            for st in states:
                self.core = st
                if self.lat is not None:
                    self.lat.begin_core(st.core_id)
                self.run_ops(seg)
            if si < len(collectives):
                self._ring_reduce(collectives[si], states)
        return self.trace

    def run_ops(self, ops: List[Operation]):
        r = None
        for op in ops:
            r = self.run_op(op)
        return r

    def run_op(self, op: Operation):
        core = self.core
        rw = self.rewrites.get(id(op))
        if rw is not None:
            res = rw(self, op)
        else:
            h = getattr(self, "op_" + op.op_type.replace(".", "_"), None)
            if h is None:
                h = _ELEMENTWISE.get(op.op_type)
                if h is None:
                    raise ValueError(f"Unknown operation: {op.op_type}")
                res = h(self, op)
            else:
                res = h(op)
        if op.results and res is not None:
            vals = res if isinstance(res, tuple) else (res,)
            if len(vals) != len(op.results):
                raise RuntimeError(
                    f"{op.op_type}: expected {len(op.results)} result(s), got {len(vals)}")
            for name, val in zip(op.results, vals):
                core.set(name, val)
                if _is_tile(val):
                    core.track(name, val.nbytes)
        if self.lat is not None:
            self._lat_record(op, res)
        return res

    # -- latency records (op-for-op with ktir_cpu/latency.py:175-265) ---------------
    def _operands(self, op):
        return [self.core.get(o) if isinstance(o, str) and self.core.has(o) else None
                for o in op.operands]

    def _lat_record(self, op, res):
        from . import latency as L
        cat = L.category(op.op_type)
        arg = None
        if cat == "memory":
            if op.op_type == "ktdp.load":
                if res.kind == "assemble":
                    arg = sum(self._load_sticks(p) for p in res.ins)
                else:
                    arg = self._load_sticks(res)
            else:
                t = self.core.get(op.operands[1])
                if isinstance(t, DistAccessV):
                    arg = sum(self._store_sticks(s.target)
                              for s in self.trace.stores[len(self.trace.stores) - len(t.pieces):])
                else:
                    arg = self._store_sticks(self.trace.stores[-1].target)
        elif cat == "compute_matmul":
            tiles = [v for v in self._operands(op) if _is_tile(v)]
            if len(tiles) >= 2:
                a, b = tiles[0].shape, tiles[1].shape
                arg = (a[0] if len(a) >= 2 else 1, b[1] if len(b) >= 2 else 1,
                       a[1] if len(a) >= 2 else a[0])
            else:
                arg = (1, 1, 1)
        elif cat != "zero":
            arg = _elements(res, self._operands(op))
        self.lat.add(op.op_type, cat, arg)

    def _load_sticks(self, n: "Node"):
        from . import latency as L
        a = n.attrs
        if a["mode"] == "indirect":
            return L.IndirectAccess(a["iat"], store=False)
        buf, isz = a["buf"], n.dtype.itemsize
        if buf.byte_base >= LX_BASE:
            return 0   # LX: no HBM traffic (ktir_cpu/latency.py:232-233)
        base = buf.byte_base + a["off"] * isz
        if a["mode"] == "rect":
            return L.rect_sticks(base, n.shape, a["strides"], isz)
        return L.coord_sticks(base, a["offsets"], isz)

    def _store_sticks(self, t):
        from . import latency as L
        if isinstance(t, IndirectTarget):
            return L.IndirectAccess(t.iat, store=True)
        isz = np.dtype(t.dtype).itemsize
        if t.buf.byte_base >= LX_BASE:
            return 0
        base = t.buf.byte_base + t.off * isz
        if isinstance(t, RectTarget):
            return L.rect_sticks(base, t.shape, t.strides, isz)
        return L.coord_sticks(base, t.offsets, isz)

    # -- inter-tile collectives ----------------------------------------------------
    def op_ktdp_inter_tile_produce(self, op):
        """This core's partial and its group (ktir_cpu/dialects/ktdp_ops.py:947-995,
        group lookup :913-940)."""
        a = op.attributes
        n = self.func.num_cores
        cid = self.core.core_id
        groups = [g for g in range(n) if a["groups"].contains([g])
                  and a["producer_tiles_per_group"].contains([cid], [g])]
        if not groups:
            raise RuntimeError(
                f"tile {cid} is not contained in any producer group "
                f"(producer_set={a['producer_tiles_per_group'].source!r}, "
                f"groups_set={a['groups'].source!r})")
        if len(groups) > 1:
            raise RuntimeError(f"tile {cid} matched multiple groups {groups} — "
                               f"violates the disjointness invariant")
        gid = groups[0]
        region = op.regions[0] if op.regions else None
        partial = None
        if region is not None:
            self.core.push()
            if region.args:
                self.core.set(region.args[0][0], gid)
            r = self.run_ops(region.ops)
            self.core.pop()
            vals = r.values if isinstance(r, _Yield) else ([r] if r is not None else [])
            partial = vals[0] if vals else None
        return FutureV(partial, a["producer_tiles_per_group"], a["groups"], gid)

    def _ring_reduce(self, op, states):
        """ktdp.inter_tile_reduce on every core at once, with the ring's fold order
        (ktir_cpu/ops/comm_ops.py:325-345): consumer c starts from its own seed
        (its partial if it produces, else its identity) and folds the seeds of
        cores c-1, c-2, ... (mod n) that produce in c's group, left to right."""
        n = len(states)
        a = op.attributes
        futs, seeds, plans = [], [], []
        for st in states:
            fut = st.get(op.operands[0])
            if not isinstance(fut, FutureV):
                raise TypeError(f"ktdp.inter_tile_reduce: operand 0 must be a TileFuture, "
                                f"got {type(fut)}")
            ident = st.get(op.operands[1]) if len(op.operands) > 1 else None
            prod = {i for i in range(n) if fut.producer_set.contains([i], [fut.group])}
            cons = {i for i in range(n) if a["consumer_tiles_per_group"].contains([i], [fut.group])}
            futs.append(fut)
            plans.append((prod, cons))
            seeds.append(fut.partial if st.core_id in prod else ident)
        region = op.regions[0] if op.regions else None
        if region is None or len(region.args) < 2:
            raise ValueError("ktdp.inter_tile_reduce: combiner region missing ^bb0 args")
        lhs, rhs = region.args[0][0], region.args[1][0]
        body = list(region.ops)
        target = a.get("result_shape")
        for st in states:
            c = st.core_id
            prod, cons = plans[c]
            self.core = st
            if self.lat is not None:
                self.lat.begin_core(c)
            acc = seeds[c]
            folds = 0
            for k in range(1, n):
                o = (c - k) % n
                if o not in prod:
                    continue
                st.push()
                st.set(lhs, acc)
                st.set(rhs, seeds[o])
                r = self.run_ops(body)
                st.pop()
                acc = r.values[0] if isinstance(r, _Yield) else r
                if not _is_tile(acc):
                    raise TypeError(f"ktdp.inter_tile_reduce: combiner did not yield a Tile, "
                                    f"got {type(acc)}")
                folds += 1
            if self.lat is not None:
                wire = (n - 1) * seeds[c].nbytes if (c in cons and _is_tile(seeds[c])) else None
                self.lat.add(op.op_type, "comm", wire)
            if c not in cons:
                # the reference hands such a core None and then fails to reshape it
                # (ktir_cpu/dialects/ktdp_helpers.py:186-189)
                raise TypeError("reshape_tile_to_target: expected Tile, got NoneType")
            if target is not None and tuple(target) != tuple(acc.shape):
                if int(np.prod(target)) != acc.numel:
                    raise ValueError(f"reshape_tile_to_target: result shape {acc.shape} and "
                                     f"declared shape {tuple(target)} have different element counts")
                acc = self.node("reshape", tuple(target), acc.dtype, (acc,), {}, acc.label)
            elif folds == 0:
                # a lone consumer gets its own seed: give the result its own node
                acc = self.node("ew", acc.shape, acc.dtype, (acc,), {"op": "cast"}, acc.label)
            if op.results:
                st.set(op.results[0], acc)
                st.track(op.results[0], acc.nbytes)

    # -- grid / views ------------------------------------------------------------
    def op_ktdp_get_compute_tile_id(self, op):
        if len(op.results) <= 1:
            return self.core.pos[0]
        return tuple(self.core.pos[d] for d in range(len(op.results)))

    def op_ktdp_construct_memory_view(self, op):
        a = op.attributes
        ptr = _need_int(self.core.get(op.operands[0]), "memory view base")
        shape = tuple(_need_int(self.core.get(s), "view size") if isinstance(s, str) else s
                      for s in a["shape"])
        strides = [_need_int(self.core.get(s), "view stride") if isinstance(s, str) else s
                   for s in a["strides"]]
        cset = a.get("coordinate_set")
        if isinstance(cset, BoxSet) and not cset.is_concrete:
            syms = tuple(int(self.core.get(s)) for s in a["shape"] if isinstance(s, str))
            cset = cset.specialize(syms)
        lx_core = None
        if a["memory_space"] == "LX":
            # a core's own scratchpad unless the view names another core's
            lx_core = a.get("lx_core_id", self.core.core_id)
        elif a["memory_space"] != "HBM":
            raise ValueError(f"Invalid memory_space {a['memory_space']!r}")
        return MemRefV(ptr, tuple(int(s) for s in shape), [int(s) for s in strides],
                       a["memory_space"], a["dtype"], cset, lx_core)

    def op_ktdp_construct_distributed_memory_view(self, op):
        """ktir_cpu/dialects/ktdp_ops.py:97-121."""
        parts = [self.core.get(o) for o in op.operands]
        for i, part in enumerate(parts):
            if not isinstance(part, MemRefV):
                raise ValueError(f"construct_distributed_memory_view: operand {i} is "
                                 f"{type(part).__name__}, expected MemRef")
        if "shape" not in op.attributes or "dtype" not in op.attributes:
            raise ValueError("construct_distributed_memory_view: missing required attributes "
                             "'shape'/'dtype'")
        dtype = op.attributes["dtype"]
        # partition checks of DistributedMemRef (ktir_cpu/ir_types.py:140-152)
        if not parts:
            raise ValueError("DistributedMemRef requires at least one partition")
        for i, part in enumerate(parts):
            if part.cset is None:
                raise ValueError(f"DistributedMemRef partition {i} must have a coordinate_set")
            if part.dtype != dtype:
                raise ValueError(f"DistributedMemRef partition {i} dtype {part.dtype!r} "
                                 f"does not match view dtype {dtype!r}")
        return DistMemRefV(parts, tuple(op.attributes["shape"]), dtype)

    def op_ktdp_construct_access_tile(self, op):
        parent = self.core.get(op.operands[0])
        idx = [_need_int(self.core.get(o), "access tile index") for o in op.operands[1:]]
        a = op.attributes
        if isinstance(parent, DistMemRefV):
            return self._dist_access(parent, idx, a)
        if not isinstance(parent, MemRefV):
            raise TypeError(f"construct_access_tile: parent is {type(parent).__name__}")
        base = a["base_map"].eval(idx)
        off = sum(int(c) * s for c, s in zip(base, parent.strides))
        cset = a["coordinate_set"]
        if isinstance(cset, BoxSet) and not cset.is_concrete:
            raise NotImplementedError("construct_access_tile: symbolic access_tile_set")
        return AccessTileV(parent.byte_address + off * bpe(parent.dtype), tuple(a["shape"]),
                           list(parent.strides), parent.dtype, cset, a.get("coordinate_order"))

    def _dist_access(self, dist: DistMemRefV, idx, a):
        """Partition routing of MemoryOps.distributed_tile_access
        (ktir_cpu/ops/memory_ops.py:651-756): C_i = B_i ∩ (x + A) per partition,
        empty intersections dropped.  Where B_i and A are both boxes C_i is a
        box; otherwise C_i is the points of B_i (enumerated over the global
        shape, in its order) that lie in x + A, and the partition's origin is
        the per-axis minimum over B_i's points."""
        x = tuple(int(v) for v in a["base_map"].eval(idx))
        shape = tuple(a["shape"])
        nd = len(shape)
        acc = a["coordinate_set"]
        xa = None
        if acc is None:
            xa = (x, tuple(x[d] + shape[d] for d in range(nd)))
        elif isinstance(acc, BoxSet) and acc.is_concrete:
            xa = (tuple(x[d] + acc.lo[d] for d in range(nd)),
                  tuple(x[d] + acc.hi[d] for d in range(nd)))
        elif isinstance(acc, BoxSet):
            raise NotImplementedError("distributed access with a symbolic access set")
        pieces = []
        for part in dist.parts:
            b = part.cset
            if isinstance(b, BoxSet) and b.is_concrete and xa is not None:
                clo = tuple(max(xa[0][d], b.lo[d]) for d in range(nd))
                chi = tuple(min(xa[1][d], b.hi[d]) for d in range(nd))
                if any(clo[d] >= chi[d] for d in range(nd)):
                    continue
                pieces.append((part, BoxSet(clo, chi), tuple(b.lo)))
                continue
            if isinstance(b, BoxSet) and not b.is_concrete:
                raise NotImplementedError("distributed view with a symbolic partition")
            pts = b.enumerate_array(tuple(dist.shape))
            if not len(pts):
                continue
            origin = tuple(int(v) for v in pts.min(0))
            rel = pts - np.asarray(x, np.int64)
            if xa is not None:
                keep = np.all((pts >= np.asarray(xa[0])) & (pts < np.asarray(xa[1])), axis=1)
            else:
                keep = np.asarray(np.broadcast_to(acc._mask(list(rel.T)), (len(pts),)), bool)
            if not keep.any():
                continue
            pieces.append((part, pts[keep], origin))
        if not pieces:
            raise ValueError(f"distributed_tile_access: no partition covers access region "
                             f"global_base={x} shape={shape}")
        return DistAccessV(x, shape, dist.dtype, pieces)

    def _points(self, part: MemRefV, pts: np.ndarray, origin, what: str):
        """(buffer, element offset, element offsets) of a partition's points
        (global coordinates), laid out by the partition's strides from its origin."""
        buf, eoff = self._resolve(part.byte_address, part.dtype, what)
        local = pts - np.asarray(origin, np.int64)
        offs = (local * np.asarray(part.strides[:pts.shape[1]], np.int64)).sum(1)
        return buf, eoff, offs

    @staticmethod
    def _positions(pts: np.ndarray, base, shape) -> np.ndarray:
        """Row-major positions, inside a tile of `shape`, of global points
        taken relative to the access origin `base`."""
        rel = pts - np.asarray(base, np.int64)
        if rel.shape[1] != len(shape) or np.any(rel < 0) or np.any(rel >= np.asarray(shape)):
            raise IndexError(f"distributed access: points outside the tile shape {shape}")
        return np.ravel_multi_index(tuple(rel.T), tuple(shape)).astype(np.int64)

    def _piece(self, part: MemRefV, box: BoxSet, origin, what: str):
        """(buffer, element offset, shape, strides) of one partition's sub-box."""
        local = [box.lo[d] - origin[d] for d in range(len(origin))]
        off = sum(l * s for l, s in zip(local, part.strides))
        buf, eoff = self._resolve(part.byte_address + off * bpe(part.dtype), part.dtype, what)
        return buf, eoff, box.extent(), tuple(part.strides[:len(origin)])

    def op_ktdp_construct_indirect_access_tile(self, op):
        a = op.attributes
        parent = self.core.get(op.operands[0])
        views = [self.core.get(o) for o in op.operands[1:]]
        consts: Dict[int, int] = {}
        for i, v in enumerate(a["var_names"]):
            if self.core.has("%" + v):
                val = self.core.get("%" + v)
                if _concrete(val):
                    consts[i] = int(val)
        shape = tuple(a["shape"])
        vss = a["variables_space_set"]
        if consts:
            if isinstance(vss, BoxSet):
                for i in consts:
                    if vss.lo[i] != 0 or vss.hi[i] > 1:
                        raise ValueError(
                            f"construct_indirect_access_tile: intermediate variable "
                            f"%{a['var_names'][i]} (index {i}) is an outer SSA value but its "
                            f"dimension in variables_space_set has a non-zero range.")
            else:
                pts = vss.enumerate_array(shape)
                for i in consts:
                    if pts.size and np.any(pts[:, i] != 0):
                        raise ValueError(
                            f"construct_indirect_access_tile: intermediate variable "
                            f"%{a['var_names'][i]} (index {i}) is an outer SSA value but its "
                            f"dimension in variables_space_set has a non-zero range.")
        refs: Dict[str, int] = {}
        for d in a["dims"]:
            for e in (d.get("exprs") or [d.get("expr")]):
                _collect_refs(e, refs)
        for r in list(refs):
            refs[r] = _need_int(self.core.get(r), "indirect subscript")
        return IATV(parent, shape, list(a["dims"]), views, vss,
                    a.get("variables_space_order"), consts, refs)

    # -- loads / stores ------------------------------------------------------------
    def _resolve(self, byte: int, dtype: str, what: str) -> Tuple[Buffer, int]:
        buf = self.space.find(byte)
        if buf is None:
            raise ValueError(f"{what} from unmapped address 0x{byte:x}")
        if buf.dtype != np_dtype(dtype):
            raise NotImplementedError(
                f"access as {dtype} to a buffer holding {buf.dtype}: reinterpreting element "
                f"types is not supported by the B200 backend")
        return buf, (byte - buf.byte_base) // bpe(dtype)

    def _coords(self, at: AccessTileV) -> np.ndarray:
        pts = at.cset.enumerate_array(at.shape)
        if at.order is not None:
            out = at.order.eval(list(pts.T))
            pts = np.stack([np.broadcast_to(np.asarray(o, np.int64), (pts.shape[0],))
                            for o in out], axis=1)
        return pts

    def op_ktdp_load(self, op):
        t = self.core.get(op.operands[0])
        rshape = op.attributes.get("result_shape")
        if isinstance(t, DistAccessV):
            # MemoryOps.distributed_load (ktir_cpu/ops/memory_ops.py:782-846): each
            # covered box read from its partition, placed into a zero tile
            shape = tuple(rshape or t.shape)
            dt = np_dtype(t.dtype)
            parts, places = [], []
            for part, box, origin in t.pieces:
                if isinstance(box, np.ndarray):
                    # scattered points: gathered in order, then placed one by one
                    buf, eoff, offs = self._points(part, box, origin, "Read")
                    parts.append(self.node("load", (len(offs),), dt, (),
                                           {"mode": "coords", "buf": buf, "off": eoff,
                                            "offsets": offs}))
                    places.append(self._positions(box, t.base, shape))
                    continue
                buf, eoff, ext, strides = self._piece(part, box, origin, "Read")
                parts.append(self.node("load", ext, dt, (), {"mode": "rect", "buf": buf,
                                                             "off": eoff, "strides": strides}))
                places.append(tuple(box.lo[d] - t.base[d] for d in range(len(shape))))
            return self.node("assemble", shape, dt, tuple(parts), {"at": places})
        if isinstance(t, IATV):
            if t.vso is not None and not t.vso.is_permutation():
                raise ValueError("indirect_load: variables_space_order must permute its input "
                                 f"dimensions; got non-permutation map: {t.vso.source}")
            pb, poff = self._resolve(t.parent.byte_address, t.parent.dtype, "Read")
            shape = tuple(rshape or t.shape)
            return self.node("load", shape, np_dtype(t.parent.dtype), (),
                             {"mode": "indirect", "iat": t, "buf": pb, "off": poff})
        if isinstance(t.cset, BoxSet) and t.order is None:
            off = sum(lo * s for lo, s in zip(t.cset.lo, t.strides))
            byte = t.byte + off * bpe(t.dtype)
            buf, eoff = self._resolve(byte, t.dtype, "Read")
            shape = t.cset.extent()
            return self.node("load", shape, np_dtype(t.dtype), (),
                             {"mode": "rect", "buf": buf, "off": eoff,
                              "strides": tuple(t.strides[:len(shape)])})
        buf, eoff = self._resolve(t.byte, t.dtype, "Read")
        coords = self._coords(t)
        offs = (coords.astype(np.int64) * np.asarray(t.strides[:coords.shape[1]], np.int64)).sum(1) \
            if coords.size else np.zeros(0, np.int64)
        shape = tuple(rshape or t.shape)
        if int(np.prod(shape)) != offs.size:
            raise ValueError(f"ktdp.load: access set has {offs.size} points but the result "
                             f"type holds {int(np.prod(shape))}")
        return self.node("load", shape, np_dtype(t.dtype), (),
                         {"mode": "coords", "buf": buf, "off": eoff, "offsets": offs})

    def op_ktdp_store(self, op):
        val = self.core.get(op.operands[0])
        if not _is_tile(val):
            raise TypeError(f"ktdp.store expects a Tile, got {type(val)}")
        t = self.core.get(op.operands[1])
        if isinstance(t, DistAccessV):
            # MemoryOps.distributed_store (ktir_cpu/ops/memory_ops.py:848-912): the
            # tile's slice over each covered box written to its partition
            for part, box, origin in t.pieces:
                if isinstance(box, np.ndarray):
                    buf, eoff, offs = self._points(part, box, origin, "Write")
                    pos = self._positions(box, t.base, tuple(val.shape))
                    sub = self.node("pick", (len(offs),), val.dtype, (val,), {"positions": pos},
                                    val.label)
                    self.trace.stores.append(Store(self.core.core_id, self.seq, sub,
                                                   CoordTarget(buf, eoff, offs, (len(offs),),
                                                               np_dtype(t.dtype)),
                                                   len(self.trace.nodes)))
                    self.seq += 1
                    continue
                buf, eoff, ext, strides = self._piece(part, box, origin, "Write")
                at = tuple(box.lo[d] - t.base[d] for d in range(len(ext)))
                sub = self.node("slice", ext, val.dtype, (val,), {"at": at}, val.label)
                self.trace.stores.append(Store(self.core.core_id, self.seq, sub,
                                               RectTarget(buf, eoff, ext, strides, np_dtype(t.dtype)),
                                               len(self.trace.nodes)))
                self.seq += 1
            return None
        if isinstance(t, IATV):
            if tuple(val.shape) != tuple(t.shape):
                raise ValueError(
                    f"indirect_store: source tile shape {tuple(val.shape)} does not match "
                    f"IAT shape {tuple(t.shape)}")
            if t.vso is not None and not t.vso.is_permutation():
                raise ValueError("indirect_store: variables_space_order must permute its input "
                                 f"dimensions; got non-permutation map: {t.vso.source}")
            self._resolve(t.parent.byte_address, t.parent.dtype, "Write")
            tgt = IndirectTarget(t)
        elif isinstance(t.cset, BoxSet) and t.order is None:
            off = sum(lo * s for lo, s in zip(t.cset.lo, t.strides))
            byte = t.byte + off * bpe(t.dtype)
            buf, eoff = self._resolve(byte, t.dtype, "Write")
            shape = t.cset.extent()
            if int(np.prod(shape)) != val.numel:
                raise ValueError(f"ktdp.store: tile of {val.numel} elements into a box of "
                                 f"{int(np.prod(shape))}")
            tgt = RectTarget(buf, eoff, shape, tuple(t.strides[:len(shape)]), np_dtype(t.dtype))
        else:
            buf, eoff = self._resolve(t.byte, t.dtype, "Write")
            coords = self._coords(t)
            offs = (coords.astype(np.int64) * np.asarray(t.strides[:coords.shape[1]], np.int64)
                    ).sum(1) if coords.size else np.zeros(0, np.int64)
            if offs.size != val.numel:
                raise ValueError(f"ktdp.store: tile of {val.numel} elements into an access set "
                                 f"of {offs.size}")
            tgt = CoordTarget(buf, eoff, offs, val.shape, np_dtype(t.dtype))
        self.trace.stores.append(Store(self.core.core_id, self.seq, val, tgt,
                                       len(self.trace.nodes)))
        self.seq += 1
        return None

    # -- constants, casts ----------------------------------------------------------
    def op_arith_constant(self, op):
        a = op.attributes
        if a.get("is_tensor"):
            dt = np_dtype(a["dtype"])
            if a.get("dense_list"):
                arr = np.array(a["value"], dtype=dt).reshape(a["shape"])
                return self.node("dense", arr.shape, dt, (), {"value": arr}, a["dtype"])
            return self.const_tile(dt.type(a["value"]), a["shape"], dt, a["dtype"])
        return a.get("value", 0)

    def _cast_to(self, v, target: np.dtype, label: str, floating: bool, name: str):
        if _is_tile(v):
            if v.dtype == target:
                return v
            cat = "f" if floating else "iu"
            if v.dtype.kind not in cat:
                raise TypeError(f"{name} expects {'float' if floating else 'integer'} Tile")
            return self.node("ew", v.shape, target, (v,), {"op": "cast"}, label)
        if isinstance(v, Node):
            if v.dtype == target and not v.pyscalar:
                return v
            return self.node("ew", (), target, (v,), {"op": "cast"}, label)
        if isinstance(v, target.type):
            return v
        r = target.type(v)
        if target.kind == "f" and np.isinf(r) and not np.isinf(float(v)):
            raise OverflowError(f"{name}: {v} overflows {target}")
        return r

    def op_arith_extf(self, op):
        v = self.core.get(op.operands[0])
        if not isinstance(v, Node):
            return np.float32(v)
        return self._cast_to(v, np.dtype(np.float32), "f32", True, "extf")

    def op_arith_convertf(self, op):
        """ArithOps.convertf (ktir_cpu/ops/arith_ops.py:660-668): f16 becomes
        f32, any other element type becomes f16."""
        v = self.core.get(op.operands[0])
        if isinstance(v, Node):
            tgt = np.dtype(np.float32 if v.dtype == np.float16 else np.float16)
            if _is_tile(v):
                return self.node("ew", v.shape, tgt, (v,), {"op": "cast"}, "convertf")
            return self.node("ew", (), tgt, (v,), {"op": "cast"}, "convertf")
        return np.float32(v) if isinstance(v, np.float16) else np.float16(v)

    def op_ktdp_coreid(self, op):
        """GridOps.coreid (ktir_cpu/ops/grid_ops.py:43-62, ktir_cpu/grid.py:
        402-470): the linear ids of the cores at grid coordinates padded with
        0 to three axes, -1 matching every position on its axis."""
        want = []
        for o in op.operands:
            v = self.core.get(o)
            if isinstance(v, Node):
                raise NotImplementedError("ktdp.coreid of a data-dependent coordinate")
            want.append(int(v))
        want = (want + [0, 0, 0])[:3]
        nx, ny, nz = self.func.grid
        out = []
        for cid in range(nx * ny * nz):
            z, r = divmod(cid, nx * ny)
            y, x = divmod(r, nx)
            if all(w == -1 or w == p for w, p in zip(want, (x, y, z))):
                out.append(cid)
        return out

    def op_arith_truncf(self, op):
        return self._cast_to(self.core.get(op.operands[0]), np.dtype(np.float16), "f16", True,
                             "truncf")

    def _int_cast(self, op, target, label):
        v = self.core.get(op.operands[0])
        if isinstance(v, Node):
            return self.node("ew", v.shape, target, (v,), {"op": "cast"}, label)
        return int(v)

    def op_arith_extsi(self, op):
        return self._int_cast(op, np.dtype(np.int64), "i64")

    op_arith_extui = op_arith_extsi

    def op_arith_trunci(self, op):
        return self._int_cast(op, np.dtype(np.int32), "i32")

    def op_arith_fptosi(self, op):
        return self._int_cast(op, np.dtype(np.int32), "i32")

    def op_arith_fptoui(self, op):
        # an unsigned tile, whatever the result type says (ops/arith_ops.py:504-508)
        return self._int_cast(op, np.dtype(np.uint32), "ui32")

    def op_arith_sitofp(self, op):
        v = self.core.get(op.operands[0])
        dst = op.attributes.get("dst_type") or (op.result_types[0] if op.result_types else "f32")
        dname = _elem(dst) or "f32"
        dt = np_dtype(dname)
        if isinstance(v, Node):
            return self.node("ew", v.shape, dt, (v,), {"op": "cast"}, dname)
        return dt.type(v)

    def op_arith_uitofp(self, op):
        v = self.core.get(op.operands[0])
        if isinstance(v, Node):
            return self.node("ew", v.shape, np.float32, (v,), {"op": "cast"}, "f32")
        return float(v)

    def op_arith_index_cast(self, op):
        v = self.core.get(op.operands[0])
        if isinstance(v, Node):
            raise DataDependentError("arith.index_cast of tile data")
        return int(v)

    op_arith_index_castui = op_arith_index_cast

    def op_arith_bitcast(self, op):
        v = self.core.get(op.operands[0])
        dst = _elem(op.attributes.get("dst_type", "f32")) or "f32"
        if isinstance(v, Node):
            return self.node("ew", v.shape, np_dtype(dst), (v,), {"op": "bitcast"}, dst)
        if dst == "f32":
            return float(np.frombuffer(int(v).to_bytes(4, "little", signed=(v < 0)),
                                       dtype=np.float32)[0])
        return int(np.frombuffer(np.float32(v).tobytes(), dtype=np.int32)[0])

    # -- elementwise arithmetic ------------------------------------------------------
    def ew(self, opname: str, operands: Sequence[Any], fn, label_from=None, attrs=None):
        """Record an elementwise op; result dtype/shape from NumPy on prototypes."""
        protos = [o.proto() if isinstance(o, Node) else o for o in operands]
        with np.errstate(all="ignore"):
            r = fn(*protos)
        rdt = np.asarray(r).dtype if not isinstance(r, (bool,)) else np.dtype(np.bool_)
        tiles = [o for o in operands if _is_tile(o)]
        if tiles:
            shape = np.broadcast_shapes(*[t.shape for t in tiles])
            pys = False
        else:
            shape = ()
            pys = isinstance(r, (float, int, bool)) and not isinstance(r, np.generic)
        ins = [o if isinstance(o, Node) else Const(o, np.asarray(o).dtype) for o in operands]
        lab = label_from.label if isinstance(label_from, Node) else None
        a = {"op": opname}
        if attrs:
            a.update(attrs)
        return self.node("ew", shape, rdt, ins, a, lab, pys)


def _elem(t: Optional[str]) -> Optional[str]:
    if not t:
        return None
    t = t.strip()
    if t.startswith("tensor<"):
        return t[len("tensor<"):-1].split("x")[-1]
    return t


def _collect_refs(e, out: dict):
    if e is None:
        return
    if e[0] == "ref":
        out[e[1]] = None
        return
    for c in e[1:]:
        if isinstance(c, tuple):
            _collect_refs(c, out)


# ---------------------------------------------------------------------------
# elementwise op handlers (registered by op name)
# ---------------------------------------------------------------------------

_ELEMENTWISE: Dict[str, Any] = {}


def _reg(*names):
    def deco(fn):
        for n in names:
            _ELEMENTWISE[n] = fn
        return fn
    return deco


_FLOAT_FN = {"arith.addf": ("add", operator.add), "arith.subf": ("sub", operator.sub),
             "arith.mulf": ("mul", operator.mul), "arith.divf": ("div", operator.truediv),
             "arith.remf": ("fmod", operator.mod)}


def _f16(tr: Tracer, v):
    """Coerce a scalar operand to float16 as the reference's float binops do."""
    if isinstance(v, Node):
        if v.dtype == np.float16 and not v.pyscalar:
            return v
        return tr.node("ew", (), np.float16, (v,), {"op": "cast"}, "f16")
    return np.float16(v)


def _float_binop(tr: Tracer, op):
    name, fn = _FLOAT_FN[op.op_type]
    a = tr.core.get(op.operands[0])
    b = tr.core.get(op.operands[1])
    if _is_scalar(a) and _is_scalar(b):
        if _concrete(a) and _concrete(b):
            with np.errstate(all="ignore"):
                r = fn(np.float16(a), np.float16(b))
            return r if isinstance(r, np.float16) else np.float16(r)
        return tr.ew(name, [_f16(tr, a), _f16(tr, b)], lambda x, y: np.float16(fn(x, y)))
    if _is_tile(a) and _is_tile(b):
        return tr.ew(name, [a, b], fn, a)
    if _is_tile(a):
        return tr.ew(name, [a, _f16(tr, b)], fn, a)
    return tr.ew(name, [_f16(tr, a), b], fn, b)


for _n in _FLOAT_FN:
    _ELEMENTWISE[_n] = _float_binop


def _truncdiv(a, b):
    return np.trunc(np.asarray(a) / np.asarray(b)).astype(np.asarray(a).dtype)


def _truncrem(a, b):
    return np.asarray(a) - _truncdiv(a, b) * np.asarray(b)


def _ceildiv_arr(a, b):
    return np.ceil(np.asarray(a) / np.asarray(b)).astype(np.result_type(a, b))


_INT_FN = {
    "arith.addi": ("add", operator.add), "arith.subi": ("sub", operator.sub),
    "arith.muli": ("mul", operator.mul), "arith.divui": ("floordiv", operator.floordiv),
    "arith.divsi": ("truncdiv", _truncdiv), "arith.floordivsi": ("floordiv", operator.floordiv),
    "arith.remui": ("mod", operator.mod), "arith.remsi": ("truncrem", _truncrem),
    "arith.ceildivsi": ("ceildiv", _ceildiv_arr), "arith.ceildivui": ("ceildiv", _ceildiv_arr),
    "arith.andi": ("and", operator.and_), "arith.ori": ("or", operator.or_),
    "arith.xori": ("xor", operator.xor), "arith.shli": ("shl", operator.lshift),
    "arith.shrsi": ("shr", operator.rshift),
}

_INT_SCALAR = {
    "arith.divsi": lambda a, b: int(np.trunc(a / b)),
    "arith.remsi": lambda a, b: a - int(np.trunc(a / b)) * b,
    "arith.ceildivsi": lambda a, b: -((-a) // b),
    "arith.ceildivui": lambda a, b: -((-a) // b),
}


def _int_binop(tr: Tracer, op):
    name, fn = _INT_FN[op.op_type]
    a = tr.core.get(op.operands[0])
    b = tr.core.get(op.operands[1])
    if _concrete(a) and _concrete(b):
        sfn = _INT_SCALAR.get(op.op_type)
        if sfn is not None and isinstance(a, int) and isinstance(b, int):
            return sfn(a, b)
        return fn(a, b)
    if isinstance(a, Node) and not _is_tile(a) and _concrete(b):
        return tr.ew(name, [a, b], fn)
    if _is_tile(a) and _is_tile(b):
        return tr.ew(name, [a, b], fn, a)
    if _is_tile(a):
        return tr.ew(name, [a, b if isinstance(b, Node) else int(b)], fn, a)
    if _is_tile(b):
        return tr.ew(name, [a if isinstance(a, Node) else int(a), b], fn, b)
    return tr.ew(name, [a, b], fn)


for _n in _INT_FN:
    _ELEMENTWISE[_n] = _int_binop


def _shrui(tr: Tracer, op):
    a = tr.core.get(op.operands[0])
    b = tr.core.get(op.operands[1])
    if _concrete(a) and _concrete(b):
        return (int(a) & 0xFFFFFFFFFFFFFFFF) >> int(b)
    return tr.ew("shru", [a, b], lambda x, y: x >> y, a if isinstance(a, Node) else None)


_ELEMENTWISE["arith.shrui"] = _shrui


_MINMAX = {"arith.maxnumf": ("fmax", np.fmax), "arith.minnumf": ("fmin", np.fmin),
           "arith.maximumf": ("maximum", np.maximum), "arith.maxf": ("maximum", np.maximum),
           "arith.minimumf": ("minimum", np.minimum), "arith.minf": ("minimum", np.minimum),
           "arith.maxsi": ("maximum", np.maximum), "arith.minsi": ("minimum", np.minimum),
           "arith.maxui": ("maximum", np.maximum), "arith.minui": ("minimum", np.minimum)}


def _minmax(tr: Tracer, op):
    name, fn = _MINMAX[op.op_type]
    a = tr.core.get(op.operands[0])
    b = tr.core.get(op.operands[1])
    if _concrete(a) and _concrete(b):
        if op.op_type in ("arith.maxsi", "arith.maxui"):
            return max(a, b)
        if op.op_type in ("arith.minsi", "arith.minui"):
            return min(a, b)
        return fn(a, b)
    ref = a if _is_tile(a) else (b if _is_tile(b) else None)
    return tr.ew(name, [a, b], fn, ref)


for _n in _MINMAX:
    _ELEMENTWISE[_n] = _minmax


@_reg("arith.negf")
def _negf(tr, op):
    v = tr.core.get(op.operands[0])
    if _concrete(v):
        return -v
    return tr.ew("neg", [v], operator.neg, v)


@_reg("arith.absf", "math.absf", "math.absi")
def _absf(tr, op):
    v = tr.core.get(op.operands[0])
    if _concrete(v):
        return abs(v)
    return tr.ew("abs", [v], np.abs, v)


_MATH = {"math.exp": "exp", "math.sqrt": "sqrt", "math.rsqrt": "rsqrt", "math.log": "log",
         "math.log2": "log2", "math.log1p": "log1p", "math.tanh": "tanh", "math.sin": "sin",
         "math.cos": "cos", "math.ceil": "ceil", "math.floor": "floor", "math.erf": "erf"}
_MATH_NP = {"exp": np.exp, "sqrt": np.sqrt, "rsqrt": lambda x: 1.0 / np.sqrt(x), "log": np.log,
            "log2": np.log2, "log1p": np.log1p, "tanh": np.tanh, "sin": np.sin, "cos": np.cos,
            "ceil": np.ceil, "floor": np.floor}


def _erf32(x):
    a = np.abs(x)
    t = 1.0 / (1.0 + 0.3275911 * a)
    poly = t * (0.254829592 + t * (-0.284496736 + t * (1.421413741 + t * (-1.453152027 +
                                                                            t * 1.061405429))))
    return np.sign(x) * (1.0 - poly * np.exp(-a * a))


@_reg(*_MATH.keys())
def _math_unary(tr, op):
    name = _MATH[op.op_type]
    v = tr.core.get(op.operands[0])
    if _concrete(v):
        if name == "erf":
            return type(v)(_erf32(np.array([float(v)]))[0])
        return type(v)(_MATH_NP[name](float(v)))
    if _is_tile(v):
        # float32 evaluation, cast back to the tile's dtype (ops/math_ops.py:30-268)
        return tr.node("ew", v.shape, v.dtype, (v,), {"op": name}, v.label)
    return tr.node("ew", (), v.dtype, (v,), {"op": name}, v.label, v.pyscalar)


@_reg("math.powf")
def _powf(tr, op):
    a = tr.core.get(op.operands[0])
    b = tr.core.get(op.operands[1])
    if _concrete(a) and _concrete(b):
        return type(a)(float(a) ** float(b))
    if not _is_tile(a):
        raise NotImplementedError("math.powf with a scalar base and tile exponent")
    return tr.node("ew", a.shape, a.dtype, (a, b if isinstance(b, Node) else Const(b, np.dtype(np.float32))),
                   {"op": "pow"}, a.label)


@_reg("math.fma")
def _fma(tr, op):
    a, b, c = (tr.core.get(o) for o in op.operands[:3])
    if _concrete(a) and _concrete(b) and _concrete(c):
        return type(a)(float(a) * float(b) + float(c))
    if not (_is_tile(a) and _is_tile(b) and _is_tile(c)):
        raise NotImplementedError("math.fma needs three tiles")
    return tr.node("ew", a.shape, a.dtype, (a, b, c), {"op": "fma"}, a.label)


def _cmp(tr, op, integer: bool):
    a = tr.core.get(op.operands[0])
    b = tr.core.get(op.operands[1])
    pred = op.attributes["predicate"]
    valid_i = {"eq", "ne", "slt", "ult", "sle", "ule", "sgt", "ugt", "sge", "uge"}
    valid_f = {"false", "true", "oeq", "olt", "ole", "ogt", "oge", "one", "ueq", "une", "ult",
               "ule", "ugt", "uge", "ord", "uno"}
    if pred not in (valid_i if integer else valid_f):
        raise NotImplementedError(f"{op.op_type}: unsupported predicate '{pred}'")
    if _concrete(a) and _concrete(b):
        return bool(_scalar_cmp(pred, a if integer else float(a), b if integer else float(b)))
    if not (_is_tile(a) or _is_tile(b)):
        raise DataDependentError("scalar comparison of tile data")
    # the reference materialises a scalar side with the tile's dtype (np.full)
    if not _is_tile(a):
        a = _splat_like(tr, a, b)
    if not _is_tile(b):
        b = _splat_like(tr, b, a)
    shape = np.broadcast_shapes(a.shape, b.shape)
    return tr.node("ew", shape, np.bool_, (a, b), {"op": "cmp", "pred": pred,
                                                   "int": integer}, "i1")


def _splat_like(tr, s, like: Node):
    if isinstance(s, Node):
        return tr.node("splat", like.shape, like.dtype, (s,), {}, like.label)
    return tr.const_tile(like.dtype.type(s), like.shape, like.dtype, like.label)


def _scalar_cmp(pred, x, y):
    nan = (x != x) or (y != y)
    return {
        "eq": x == y, "ne": x != y, "slt": x < y, "ult": x < y, "sle": x <= y, "ule": x <= y,
        "sgt": x > y, "ugt": x > y, "sge": x >= y, "uge": x >= y,
        "false": False, "true": True, "oeq": x == y, "olt": x < y, "ole": x <= y,
        "ogt": x > y, "oge": x >= y, "one": (x != y) and not nan, "ueq": (x == y) or nan,
        "une": x != y, "ult_": 0, "ord": not nan, "uno": nan,
    }.get(pred, None) if pred not in ("ult", "ule", "ugt", "uge") or isinstance(x, int) else \
        {"ult": (x < y) or nan, "ule": (x <= y) or nan, "ugt": (x > y) or nan,
         "uge": (x >= y) or nan}[pred]


_ELEMENTWISE["arith.cmpi"] = lambda tr, op: _cmp(tr, op, True)
_ELEMENTWISE["arith.cmpf"] = lambda tr, op: _cmp(tr, op, False)


@_reg("arith.select")
def _select(tr, op):
    c = tr.core.get(op.operands[0])
    t = tr.core.get(op.operands[1])
    f = tr.core.get(op.operands[2])
    if _concrete(c):
        return t if c else f
    if not _is_tile(c):
        raise DataDependentError("arith.select on a scalar extracted from tile data")
    ref = t if _is_tile(t) else f
    lab = ref.label if _is_tile(ref) else "f16"
    return _select_node(tr, c, t, f, lab)


def _select_node(tr, c, t, f, label):
    protos = [o.proto() if isinstance(o, Node) else o for o in (c, t, f)]
    rdt = np.asarray(np.where(*protos)).dtype
    tiles = [o for o in (c, t, f) if _is_tile(o)]
    shape = np.broadcast_shapes(*[x.shape for x in tiles])
    ins = [o if isinstance(o, Node) else Const(o, np.asarray(o).dtype) for o in (c, t, f)]
    return tr.node("ew", shape, rdt, ins, {"op": "select"}, label)


# ---------------------------------------------------------------------------
# tensor / linalg / scf handlers (methods attached to Tracer)
# ---------------------------------------------------------------------------

def _op_tensor_empty(self, op):
    a = op.attributes
    dt = np_dtype(a["dtype"])
    return self.const_tile(dt.type(0), a["shape"], dt, a["dtype"])


def _op_tensor_splat(self, op):
    s = self.core.get(op.operands[0])
    shape = tuple(op.attributes.get("shape", ())) or (1,)
    dname = op.attributes.get("dtype", "f16")
    if _is_tile(s):
        s = self.node("extract", (), s.dtype, (s,), {"index": (0,) * len(s.shape)}, s.label)
    is_int = (isinstance(s, (int, np.integer)) and not isinstance(s, (bool, np.bool_))) or \
        (isinstance(s, Node) and s.dtype.kind in "iu")
    dt = np.dtype(np.int32) if is_int else np_dtype(dname)
    lab = "i32" if is_int else dname
    if isinstance(s, Node):
        return self.node("splat", shape, dt, (s,), {}, lab)
    with np.errstate(all="ignore"):
        return self.const_tile(np.full((), s, dtype=dt)[()], shape, dt, lab)


def _op_tensor_extract(self, op):
    src = self.core.get(op.operands[0])
    if _is_tile(src):
        idx = tuple(_need_int(self.core.get(o), "tensor.extract index") for o in op.operands[1:])
        if not idx:
            idx = (0,) * len(src.shape)
        return self.node("extract", (), src.dtype, (src,), {"index": idx}, src.label)
    return src


def _op_reshape(self, op):
    src = self.core.get(op.operands[0])
    ts = op.attributes.get("target_shape")
    if _is_tile(src) and ts:
        if int(np.prod(ts)) != src.numel:
            raise ValueError(f"cannot reshape {src.shape} into {ts}")
        return self.node("reshape", tuple(ts), src.dtype, (src,), {}, src.label)
    return src


def _op_tensor_from_elements(self, op):
    vals = [self.core.get(o) for o in op.operands]
    a = op.attributes
    if all(_concrete(v) for v in vals):
        arr = np.array(vals, dtype=np_dtype(a["dtype"])).reshape(a["shape"])
        return self.node("dense", arr.shape, arr.dtype, (), {"value": arr}, a["dtype"])
    raise DataDependentError("tensor.from_elements of tile data")


def _op_tensor_generate(self, op):
    a = op.attributes
    shape = tuple(a["shape"])
    region = op.regions[0]
    self.core.push()
    for d, (name, _) in enumerate(region.args):
        rs = [1] * len(shape)
        rs[d] = shape[d]
        io = self.node("iota", tuple(rs), np.int64, (), {"dim": d}, "index")
        self.core.set(name, self.node("bcast", shape, np.int64, (io,),
                                      {"map": tuple(range(len(shape)))}, "index"))
    r = self.run_ops(region.ops)
    if isinstance(r, _Yield):
        r = r.values[0]
    self.core.pop()
    dt = np_dtype(a["dtype"])
    if isinstance(r, Node):
        if r.shape != shape:
            r = _bcast_to(self, r, shape)
        return self.node("ew", shape, dt, (r,), {"op": "cast"}, a["dtype"]) if r.dtype != dt else r
    return self.const_tile(dt.type(r), shape, dt, a["dtype"])


def _yield(self, op):
    return _Yield([self.core.get(o) for o in op.operands])


def _op_return(self, op):
    return self.core.get(op.operands[0]) if op.operands else None


def _bcast_to(tr, v: Node, shape):
    """NumPy broadcasting of v (aligned right) to shape."""
    nd = len(shape)
    off = nd - len(v.shape)
    return tr.node("bcast", shape, v.dtype, (v,), {"map": tuple(range(off, nd))}, v.label)


def _region_fold(tr, t: Node, dim, region, names) -> Node:
    """linalg.reduce with a multi-op combiner region, folded the way the
    reference folds it (ktir_cpu/dialects/linalg_ops.py:60-133, 196-207):
    each round runs the region once on the two halves of the reduced axis
    (first half bound to the first block argument, second half to the
    second), an odd leftover slice is carried into the next round, and the
    axis of extent 1 is squeezed at the end.  The region's ops become
    ordinary graph nodes over slices of the running accumulator, so the
    generic executor runs the fold; a name the region reads but the block
    arguments do not bind fails here as it does in the reference."""
    acc = t
    if dim is None:
        acc = tr.node("reshape", (t.numel,), t.dtype, (t,), {}, t.label)
        dim = 0
    n = acc.shape[dim]

    def part(src, lo, hi):
        shape = tuple(hi - lo if i == dim else s for i, s in enumerate(src.shape))
        at = tuple(lo if i == dim else 0 for i in range(len(src.shape)))
        return tr.node("slice", shape, src.dtype, (src,), {"at": at}, src.label)

    lat, tr.lat = tr.lat, None   # the fold's latency is charged by _lat_fold
    try:
        return _region_rounds(tr, t, acc, dim, n, region, names, part)
    finally:
        tr.lat = lat


def _region_rounds(tr, t, acc, dim, n, region, names, part) -> Node:
    while n > 1:
        h = n // 2
        tr.core.push()
        try:
            if names:
                tr.core.set(names[0], part(acc, 0, h))
            if len(names) > 1:
                tr.core.set(names[1], part(acc, h, 2 * h))
            r = tr.run_ops(list(region.ops))
        finally:
            tr.core.pop()
        c = r.values[0] if isinstance(r, _Yield) else r
        if not _is_tile(c):
            # the reference's fold takes the extent of the 0-d result along the
            # reduced axis (ktir_cpu/dialects/linalg_ops.py:124-131), which fails
            raise IndexError("linalg.reduce: the combiner region yields a scalar, which has "
                             "no extent along the reduced dimension")
        if n % 2:
            # the odd slice joins the combined one as NumPy's concatenate joins
            # them: both in the wider of the two element types
            tail = part(acc, 2 * h, n)
            dt = np.result_type(c.dtype, tail.dtype)
            if c.dtype != dt:
                c = tr.node("ew", c.shape, dt, (c,), {"op": "cast"}, t.label)
            if tail.dtype != dt:
                tail = tr.node("ew", tail.shape, dt, (tail,), {"op": "cast"}, t.label)
            shape = tuple(h + 1 if i == dim else s for i, s in enumerate(c.shape))
            tail_at = tuple(h if i == dim else 0 for i in range(len(shape)))
            c = tr.node("assemble", shape, dt, (c, tail),
                        {"at": [(0,) * len(shape), tail_at]}, t.label)
        acc = c
        n = h + (n % 2)
    if acc.dtype != t.dtype:
        # a combiner that changes the element type: the folded value is cast
        # back to the input's type (linalg_ops.py:196-204)
        acc = tr.node("ew", acc.shape, t.dtype, (acc,), {"op": "cast"}, t.label)
    shape = tuple(s for i, s in enumerate(acc.shape) if i != dim)
    return tr.node("reshape", shape, t.dtype, (acc,), {}, t.label, pyscalar=not shape)


def _op_linalg_reduce(self, op):
    t = self.core.get(op.operands[0])
    a = op.attributes
    if op.regions and op.regions[0].ops:
        region = op.regions[0]
        body = [o for o in region.ops if o.op_type != "linalg.yield"]
        names = linalg_block_args(region)
        if len(body) != 1 or list(body[0].operands[:2]) not in (names[:2], names[:2][::-1]):
            comb = ("region", region, names)
        else:
            comb = body[0].op_type
            if list(body[0].operands[:2]) == names[:2][::-1]:
                comb = ("swapped", comb)
    else:
        comb = a.get("combiner") or "arith.addf"
    dims = a.get("dims")
    if not _is_tile(t):
        res = t
    elif isinstance(comb, tuple) and comb[0] == "region":
        res = _region_fold(self, t, dims[0] if dims else None, comb[1], comb[2])
    else:
        dim = dims[0] if dims else None
        if dim is None:
            flat = self.node("reshape", (t.numel,), t.dtype, (t,), {}, t.label)
            res = self.node("reduce", (), t.dtype, (flat,), {"dim": 0, "combiner": comb},
                            t.label, pyscalar=True)
        else:
            shape = tuple(s for i, s in enumerate(t.shape) if i != dim)
            res = self.node("reduce", shape, t.dtype, (t,), {"dim": dim, "combiner": comb},
                            t.label, pyscalar=not shape)
    if self.lat is not None and _is_tile(t):
        _lat_fold(self, op, t, dims[0] if dims else None)
    outs = a.get("outs")
    if outs and res is not None:
        self.core.set(outs, res)
    return res


def _lat_fold(self, op, t: Node, dim):
    """Latency records of the pairwise tree fold: the combiner region runs once
    per round on halves of the reduced axis (ktir_cpu/dialects/linalg_ops.py:
    84-133), each of its ops charged on the half-size operands."""
    from . import latency as L
    if op.regions and op.regions[0].ops:
        region = op.regions[0]
        body = list(region.ops)
        names = linalg_block_args(region)
    else:
        fn = op.attributes.get("combiner") or "arith.addf"
        body = [Operation(fn, ["__comb__"], ["__in__", "__acc__"], {}),
                Operation("linalg.yield", [], ["__comb__"], {})]
        names = ["__in__", "__acc__"]
    shape = list(t.shape) if dim is not None else [t.numel]
    d = dim if dim is not None else 0
    n = shape[d]
    while n > 1:
        half = n // 2
        shape[d] = half
        elems = int(np.prod(shape))
        tiles = set(names[:2])
        for o in body:
            cat = L.category(o.op_type)
            on_tile = any(x in tiles for x in o.operands)
            if on_tile:
                tiles.update(o.results)
            if cat == "compute_matmul":
                arg = (1, 1, 1)
            elif cat == "zero":
                arg = None
            else:
                arg = elems if on_tile else 1
            self.lat.add(o.op_type, cat, arg)
        n = half + n % 2


def _op_linalg_add(self, op):
    x = self.core.get(op.operands[0])
    y = self.core.get(op.operands[1])
    return self.ew("add", [x, y], operator.add, x)


def _op_linalg_fill(self, op):
    s = self.core.get(op.operands[0])
    o = self.core.get(op.operands[1])
    if isinstance(s, Node):
        return self.node("splat", o.shape, o.dtype, (self.node("ew", (), np.float64, (s,),
                                                               {"op": "cast"}),), {}, o.label)
    return self.const_tile(o.dtype.type(float(s)), o.shape, o.dtype, o.label)


def _op_linalg_broadcast(self, op):
    x = self.core.get(op.operands[0])
    o = self.core.get(op.operands[1])
    dims = sorted(op.attributes.get("dimensions", []))
    keep = [d for d in range(len(o.shape)) if d not in dims]
    return self.node("bcast", o.shape, x.dtype, (x,), {"map": tuple(keep)}, x.label)


def _op_linalg_matmul(self, op):
    x = self.core.get(op.operands[0])
    y = self.core.get(op.operands[1])
    if len(x.shape) != 2 or len(y.shape) != 2 or x.shape[1] != y.shape[0]:
        raise ValueError(f"linalg.matmul shape mismatch {x.shape} @ {y.shape}")
    rdt = np.matmul(x.proto(), y.proto()).dtype
    mm = self.node("matmul", (x.shape[0], y.shape[1]), x.dtype, (x, y),
                   {"acc_dtype": rdt}, x.label)
    if len(op.operands) > 2:
        acc = self.core.get(op.operands[2])
        if _is_tile(acc):
            r = self.ew("add", [acc, mm], operator.add, acc)
            r.attrs["matmul_accumulate"] = True
            return r
    return mm


def _op_linalg_batch_matmul(self, op):
    x = self.core.get(op.operands[0])
    y = self.core.get(op.operands[1])
    rdt = np.matmul(x.proto(), y.proto()).dtype
    shape = tuple(np.broadcast_shapes(x.shape[:-2], y.shape[:-2])) + (x.shape[-2], y.shape[-1])
    mm = self.node("matmul", shape, rdt, (x, y), {"acc_dtype": rdt, "batched": True}, x.label)
    if len(op.operands) > 2:
        acc = self.core.get(op.operands[2])
        if _is_tile(acc):
            return self.ew("add", [acc, mm], operator.add, acc)
    return mm


def _op_linalg_transpose(self, op):
    x = self.core.get(op.operands[0])
    perm = tuple(op.attributes["permutation"])
    return self.node("transpose", tuple(x.shape[i] for i in perm), x.dtype, (x,),
                     {"perm": perm}, x.label)


def _op_linalg_generic(self, op):
    a = op.attributes
    n_ins = a["n_ins"]
    maps = a["indexing_maps"]
    ins = [self.core.get(o) for o in op.operands[:n_ins]]
    outs = self.core.get(op.operands[n_ins])
    region = op.regions[0]
    names = linalg_block_args(region)
    shape = outs.shape
    self.core.push()
    self.core.set("__linalg_shape__", shape)
    for i, (v, m) in enumerate(zip(ins, maps[:n_ins])):
        dims = tuple(e[1] for e in m.exprs if e[0] == "d")
        if _is_tile(v):
            if len(dims) != len(v.shape):
                raise NotImplementedError("linalg.generic indexing map with non-dim results")
            arg = self.node("bcast", shape, v.dtype, (v,), {"map": dims}, v.label)
        else:
            arg = v
        if i < len(names):
            self.core.set(names[i], arg)
    if n_ins < len(names):
        self.core.set(names[n_ins], outs)
    r = self.run_ops(region.ops)
    self.core.pop()
    if isinstance(r, _Yield):
        r = r.values[0] if len(r.values) == 1 else r.values[0]
    if isinstance(r, Node):
        if r.shape != shape:
            r = _bcast_to(self, r, shape) if r.shape else self.node("splat", shape, r.dtype, (r,),
                                                                     {}, r.label)
        if r.dtype != outs.dtype:
            r = self.node("ew", shape, outs.dtype, (r,), {"op": "cast"}, outs.label)
        else:
            r.label = outs.label
        return r
    with np.errstate(all="ignore"):
        return self.const_tile(np.full((), r, dtype=outs.dtype)[()], shape, outs.dtype, outs.label)


def _op_linalg_index(self, op):
    d = op.attributes["dim"]
    shape = self.core.get("__linalg_shape__")
    rs = [1] * len(shape)
    rs[d] = shape[d]
    return self.node("iota", tuple(rs), np.int64, (), {"dim": d}, "index")


def _op_scf_for(self, op):
    lb, ub, st = (_need_int(self.core.get(o), "scf.for bound") for o in op.operands[:3])
    names = op.attributes.get("iter_args", [])
    cur = [self.core.get(o) for o in op.operands[3:]]
    for n, v in zip(names, cur):
        self.core.set(n, v)
        if _is_tile(v):
            self.core.track(n, v.nbytes)
    body = op.regions[0]
    iv = op.attributes["iter_var"]
    for i in range(lb, ub, max(st, 1)):
        self.core.push()
        self.core.set(iv, i)
        r = self.run_ops(body.ops)
        ys = r.values if isinstance(r, _Yield) and names else None
        self.core.pop()
        if ys is not None:
            for n, v in zip(names, ys):
                self.core.untrack(n)
                self.core.set(n, v)
                if _is_tile(v):
                    self.core.track(n, v.nbytes)
            cur = list(ys)
    if not cur:
        return None
    return cur[0] if len(cur) == 1 else tuple(cur)


def _op_scf_if(self, op):
    c = self.core.get(op.operands[0])
    if isinstance(c, Node):
        raise DataDependentError("scf.if on tile data")
    region = op.regions[0] if c else (op.regions[1] if len(op.regions) > 1 else None)
    if region is None or not region.ops:
        return None
    self.core.push()
    r = self.run_ops(region.ops)
    self.core.pop()
    if isinstance(r, _Yield):
        if not r.values:
            return None
        return r.values[0] if len(r.values) == 1 else tuple(r.values)
    return r


for _name, _fn in list(globals().items()):
    if _name.startswith("_op_"):
        setattr(Tracer, "op_" + _name[4:], _fn)
Tracer.op_tensor_expand_shape = _op_reshape
Tracer.op_tensor_collapse_shape = _op_reshape
Tracer.op_tensor_reshape = _op_reshape
Tracer.op_tensor_yield = _yield
Tracer.op_linalg_yield = _yield
Tracer.op_scf_yield = _yield
Tracer.op_ktdp_yield_partial = _yield
Tracer.op_ktdp_yield_reduced = _yield
