"""CPU oracle: a NumPy restatement of the ktir-cpu interpreter's execution path.

TEST INFRASTRUCTURE ONLY.  This module is the checker the B200 backend is
compared against (and the timed CPU baseline in ``bench.py``).  Nothing in
the ``ktir_cpu_b200`` product imports or calls it; the product path fails
loudly when its CUDA library is missing instead of falling back here.

What it restates (reference file:line for each rule):

* cores run one after another in linear-id order, x fastest
  (ktir_cpu/grid.py:402-416, 542-560) — core k sees every HBM write of
  cores < k;
* HBM is a sparse, stick-addressed byte space (128-byte sticks, allocations
  from 0x10000, stick-aligned bump; ktir_cpu/memory.py:201-288).  A read
  resolves the allocation containing its start address and zero-pads past
  that allocation's end; a write truncates at it (memory.py:97-198);
* rectangular loads/stores take the sub-tile fast path for box access sets
  with identity order (dialects/ktdp_ops.py:181-241), contiguous or strided
  (ops/memory_ops.py:438-587); other access sets enumerate coordinates and
  gather / read-modify-write scatter with last-writer-wins;
* indirect access tiles enumerate the variable space (row-major, or sorted
  by a permutation ``variables_space_order``), read index values, reject
  negative indices with IndexError, then gather / scatter
  (ops/memory_ops.py:170-309, 589-630, 914-966; dialects/ktdp_ops.py:584-732);
* float binops coerce scalar operands to float16 (dialects/_helpers.py:35-54);
  math ops compute in float32 and cast back (ops/math_ops.py:30-268);
* linalg.reduce folds the combiner region pairwise, halving the axis and
  carrying an odd tail (dialects/linalg_ops.py:86-219);
* linalg.matmul = outs + np.matmul(a, b).astype(a.dtype)
  (dialects/linalg_ops.py:273-319, ops/arith_ops.py:403-419);
* LX accounting: every Tile-valued result is charged to the core's 2 MiB
  scratchpad, freed when its region scope pops; overflow raises
  MemoryError("LX scratchpad overflow ...") (grid.py:204-311,
  interpreter.py:216-226, ops/control_ops.py:77-167).

Unlike the reference memory simulator it does not flatten and copy a whole
allocation on every access (memory.py:131-198); reads and writes touch only
the addressed span, which changes its speed, not its results.
"""

from __future__ import annotations

import bisect
import math
import operator
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from ktir_cpu_b200.affine import BoxSet, eval_expr
from ktir_cpu_b200.ir import IRModule, Operation, Region, linalg_block_args
from ktir_cpu_b200.parser import KTIRParser

STICK = 128
LX_CAPACITY = 2 * 1024 * 1024

NP_DTYPES = {
    "f16": np.float16, "fp16": np.float16, "float16": np.float16,
    "f32": np.float32, "float32": np.float32,
    "i1": np.bool_, "i32": np.int32, "si32": np.int32, "index": np.int32,
    "i64": np.int64, "si64": np.int64,
}
KTIR_OF = {np.dtype(np.float16): "f16", np.dtype(np.float32): "f32",
           np.dtype(np.int32): "i32", np.dtype(np.int64): "i64"}


def np_dtype(name: str):
    if name in ("fp8", "mxfp8"):
        raise NotImplementedError(f"dtype {name!r} is a placeholder")
    try:
        return NP_DTYPES[name]
    except KeyError:
        raise ValueError(f"Unsupported KTIR dtype: {name!r}")


def bpe(name: str) -> int:
    return np.dtype(np_dtype(name)).itemsize


# ---------------------------------------------------------------------------
# values
# ---------------------------------------------------------------------------

@dataclass
class Tile:
    data: np.ndarray
    dtype: str
    shape: Tuple[int, ...]

    def nbytes(self) -> int:
        return self.data.nbytes


@dataclass
class MemRef:
    base: int                 # stick index (HBM)
    shape: Tuple[int, ...]
    strides: List[int]
    space: str
    dtype: str
    coordinate_set: Any = None

    @property
    def byte_address(self) -> int:
        return self.base * STICK if self.space == "HBM" else self.base


@dataclass
class TileRef:
    byte: int
    shape: Tuple[int, ...]
    strides: List[int]
    dtype: str
    space: str


@dataclass
class AccessTile:
    ref: TileRef
    shape: Tuple[int, ...]
    cset: Any
    order: Any


@dataclass
class DistRef:
    """A distributed memory view: partitions whose coordinate sets are in global
    coordinates (ktir_cpu/ir_types.py:122-152)."""
    parts: List[MemRef]
    shape: Tuple[int, ...]
    dtype: str


@dataclass
class DistTile:
    """An access tile over a distributed view, routed to the partitions it
    covers: (partition, covered set C_i, partition origin p_i); C_i is a
    (lo, hi) box or an (N, ndim) array of global points."""
    base: Tuple[int, ...]
    shape: Tuple[int, ...]
    survivors: List[Tuple[MemRef, Any, Tuple[int, ...]]]


@dataclass
class IndirectTile:
    parent: MemRef
    shape: Tuple[int, ...]
    dims: List[dict]
    views: List[MemRef]
    vss: Any
    vso: Any
    consts: Dict[int, int]    # intermediate-variable index -> bound outer SSA value


@dataclass
class _Future:
    partial: Any
    producer_set: Any
    group: int


class _Yield:
    __slots__ = ("values",)

    def __init__(self, values):
        self.values = values


# ---------------------------------------------------------------------------
# HBM simulator (sparse, allocation-bounded reads/writes)
# ---------------------------------------------------------------------------

class HBM:
    def __init__(self) -> None:
        self.allocs: Dict[int, np.ndarray] = {}
        self._starts: List[int] = []
        self.next_ptr = 0x10000

    def allocate(self, nbytes: int) -> int:
        ptr = self.next_ptr
        self.next_ptr = (ptr + nbytes + STICK - 1) & ~(STICK - 1)
        return ptr // STICK

    def _find(self, addr: int):
        if addr in self.allocs:
            return addr, self.allocs[addr]
        k = bisect.bisect_right(self._starts, addr) - 1
        if k >= 0:
            base = self._starts[k]
            arr = self.allocs[base]
            if base < addr < base + arr.nbytes:
                return base, arr
        return None

    def read_bytes(self, addr: int, n: int, dtype: str) -> np.ndarray:
        """n elements of `dtype` from byte address addr; zero past the allocation end."""
        found = self._find(addr)
        if found is None:
            raise ValueError(f"Read from unmapped address 0x{addr:x} (n_elements={n})")
        base, arr = found
        off = (addr - base) // bpe(dtype)
        out = np.zeros(n, dtype=np_dtype(dtype))
        avail = max(0, min(n, arr.size - off))
        if avail:
            out[:avail] = arr[off:off + avail]
        return out

    def write_bytes(self, addr: int, data: np.ndarray) -> None:
        found = self._find(addr)
        flat = np.ascontiguousarray(data).reshape(-1)
        if found is None:
            self.allocs[addr] = flat.copy()
            bisect.insort(self._starts, addr)
            return
        base, arr = found
        off = (addr - base) // flat.itemsize
        fit = max(0, min(flat.size, arr.size - off))
        arr[off:off + fit] = flat[:fit]

    # stick façade used by callers that seed memory directly
    def read(self, stick: int, n: int, dtype: str, *, intra_byte: int = 0) -> np.ndarray:
        return self.read_bytes(stick * STICK + intra_byte, n, dtype)

    def write(self, stick: int, data: np.ndarray, *, intra_byte: int = 0) -> None:
        self.write_bytes(stick * STICK + intra_byte, data)

    def read_gather(self, addr: int, offsets: np.ndarray, dtype: str) -> np.ndarray:
        """Elements at addr + offsets*bpe, all resolved in addr's allocation (zero past its end)."""
        if offsets.size == 0:
            return np.zeros(0, dtype=np_dtype(dtype))
        span = int(offsets.max()) + 1
        flat = self.read_bytes(addr, span, dtype)
        return flat[offsets]

    def scatter(self, addr: int, offsets: np.ndarray, values: np.ndarray, dtype: str) -> None:
        """Read-modify-write over the span starting at addr; duplicate offsets: last wins."""
        if offsets.size == 0:
            return
        span = int(offsets.max()) + 1
        flat = self.read_bytes(addr, span, dtype)
        flat[offsets] = values.reshape(-1).astype(flat.dtype, copy=False)
        self.write_bytes(addr, flat)


# ---------------------------------------------------------------------------
# per-core context: scoped SSA values + LX accounting
# ---------------------------------------------------------------------------

class Core:
    def __init__(self, core_id: int, pos: Tuple[int, int, int]):
        self.core_id = core_id
        self.pos = pos
        self.scopes: List[Dict[str, Any]] = [{}]
        self.lx_used = 0
        self.lx_bytes: Dict[str, int] = {}

    def push(self):
        self.scopes.append({})

    def pop(self):
        scope = self.scopes.pop()
        for name in scope:
            self.untrack(name)

    def set(self, name, value):
        self.scopes[-1][name] = value

    def get(self, name):
        for s in reversed(self.scopes):
            if name in s:
                return s[name]
        raise KeyError(f"Value '{name}' not found in core {self.core_id}")

    def has(self, name) -> bool:
        return any(name in s for s in self.scopes)

    def track(self, name, size):
        if self.lx_used + size > LX_CAPACITY:
            raise MemoryError(
                f"LX scratchpad overflow on core {self.core_id}: requested {size} bytes, "
                f"available {LX_CAPACITY - self.lx_used} bytes (capacity {LX_CAPACITY} bytes)")
        self.lx_bytes[name] = size
        self.lx_used += size

    def untrack(self, name):
        if name in self.lx_bytes:
            self.lx_used -= self.lx_bytes.pop(name)


def _is_scalar(v) -> bool:
    return isinstance(v, (int, float, bool, np.integer, np.floating, np.bool_))


def _contiguous(shape, strides) -> bool:
    expect = 1
    for d, s in zip(reversed(shape), reversed(strides)):
        if s != expect:
            return False
        expect *= d
    return True


def _offsets(shape, strides, coords: Optional[np.ndarray] = None) -> np.ndarray:
    st = np.asarray(strides[:len(shape)], dtype=np.int64)
    if coords is None:
        if 0 in shape:
            return np.zeros(0, dtype=np.int64)
        grids = np.indices(shape, dtype=np.int64).reshape(len(shape), -1)
        return (grids * st[:, None]).sum(axis=0)
    if coords.size == 0:
        return np.zeros(0, dtype=np.int64)
    return (coords.astype(np.int64) * np.asarray(strides[:coords.shape[1]], np.int64)).sum(axis=1)


# ---------------------------------------------------------------------------
# interpreter
# ---------------------------------------------------------------------------

class OracleInterpreter:
    """Sequential NumPy executor of a parsed KTIR function."""

    def __init__(self) -> None:
        self.module: Optional[IRModule] = None
        self.hbm: Optional[HBM] = None
        self.grid: Tuple[int, int, int] = (1, 1, 1)
        self.core_limit: Optional[int] = None   # run only the first k cores (bounded CPU samples)
        # (stick, array) pairs written into HBM before the call's arguments,
        # for programs that address memory through constants
        self.preload: List[Tuple[int, np.ndarray]] = []
        # run only the first k iterations of each core's outermost scf.for
        # (bounded CPU samples); loop_fraction records the share of that
        # loop's iterations that ran
        self.loop_limit: Optional[int] = None
        self.loop_fraction = 1.0
        self._for_depth = 0

    def load(self, src: str) -> None:
        p = KTIRParser()
        if "\n" in src or src.lstrip().startswith("module"):
            self.module = p.parse_module(src)
        else:
            self.module = p.parse_file(src)

    def execute_function(self, func_name: str, **kwargs) -> Dict[str, np.ndarray]:
        if self.module is None:
            raise RuntimeError("No module loaded. Call load() first.")
        fn = self.module.get_function(func_name)
        self.grid = fn.grid
        self.hbm = HBM()
        for stick, arr in self.preload:
            self.hbm.write(stick, np.array(arr, copy=True))
        declared = fn.arg_names
        if kwargs and declared and not any(k in declared for k in kwargs):
            if len(kwargs) == len(declared):
                kwargs = dict(zip(declared, kwargs.values()))
        ptrs: Dict[str, Any] = {}
        dts: Dict[str, str] = {}
        for name, v in kwargs.items():
            if isinstance(v, np.ndarray):
                stick = self.hbm.allocate(v.nbytes)
                self.hbm.write(stick, v)
                ptrs[name] = stick
                dts[name] = KTIR_OF[np.dtype(v.dtype)]
            else:
                ptrs[name] = v
        nx, ny, nz = fn.grid
        n = nx * ny * nz
        self.n_cores = n
        limit = n if self.core_limit is None else min(n, self.core_limit)
        cores = []
        for cid in range(limit):
            z, r = divmod(cid, nx * ny)
            y, x = divmod(r, nx)
            core = Core(cid, (x, y, z))
            for aname, _ in fn.arguments:
                key = aname.lstrip("%")
                if key in ptrs:
                    core.set(aname, ptrs[key])
            cores.append(core)
        # Top-level ktdp.inter_tile_reduce ops are collectives: every core runs
        # up to one, the ring runs, every core continues (the order the
        # reference's scheduler produces, ktir_cpu/grid.py:471-570).
        segments, collectives = [[]], []
        for op in fn.operations:
            if op.op_type == "ktdp.inter_tile_reduce":
                collectives.append(op)
                segments.append([])
            else:
                segments[-1].append(op)
        for si, seg in enumerate(segments):
            for core in cores:
                self.run_ops(core, seg)
            if si < len(collectives):
                self._ring(collectives[si], cores)
        out = {}
        for name, v in kwargs.items():
            if isinstance(v, np.ndarray):
                out[name] = self.hbm.read(ptrs[name], v.size, dts[name]).reshape(v.shape)
        return out

    # -- dispatch ------------------------------------------------------------
    def run_ops(self, core: Core, ops: List[Operation]):
        result = None
        for op in ops:
            result = self.run_op(core, op)
        return result

    def run_op(self, core: Core, op: Operation):
        h = getattr(self, "op_" + op.op_type.replace(".", "_"), None)
        if h is None:
            if op.op_type.startswith("arith.") or op.op_type.startswith("math."):
                h = self._elementwise_handler(op.op_type)
            if h is None:
                raise ValueError(f"Unknown operation: {op.op_type}")
        res = h(core, op)
        if op.results and res is not None:
            vals = res if isinstance(res, tuple) else (res,)
            if len(vals) != len(op.results):
                raise RuntimeError(
                    f"{op.op_type}: expected {len(op.results)} result(s), got {len(vals)}")
            for name, val in zip(op.results, vals):
                core.set(name, val)
                if isinstance(val, Tile):
                    core.track(name, val.nbytes())
        return res

    def run_region(self, core: Core, region: Region):
        return self.run_ops(core, region.ops)

    # -- inter-tile produce / ring reduce ----------------------------------------------
    def op_ktdp_inter_tile_produce(self, core, op):
        """ktir_cpu/dialects/ktdp_ops.py:947-995 with the group lookup of :913-940."""
        a = op.attributes
        n = self.n_cores
        keys = [g for g in range(n) if a["groups"].contains([g])
                and a["producer_tiles_per_group"].contains([core.core_id], [g])]
        if len(keys) != 1:
            raise RuntimeError(f"tile {core.core_id} matched groups {keys}")
        gid = keys[0]
        region = op.regions[0]
        core.push()
        if region.args:
            core.set(region.args[0][0], gid)
        r = self.run_ops(core, region.ops)
        core.pop()
        part = r.values[0] if isinstance(r, _Yield) else r
        return _Future(part, a["producer_tiles_per_group"], gid)

    def op_ktdp_yield_partial(self, core, op):
        return _Yield([core.get(o) for o in op.operands])

    op_ktdp_yield_reduced = op_ktdp_yield_partial

    def _ring(self, op, cores):
        """RingReduceBackend.run (ktir_cpu/ops/comm_ops.py:283-345) for every core:
        the tile core c receives in round k comes from core (c - k) mod n and is
        folded into c's accumulator when that core produces in c's group."""
        n = self.n_cores
        a = op.attributes
        region = op.regions[0]
        lhs, rhs = region.args[0][0], region.args[1][0]
        info = []
        for core in cores:
            fut = core.get(op.operands[0])
            part, pset, gid = fut.partial, fut.producer_set, fut.group
            ident = core.get(op.operands[1]) if len(op.operands) > 1 else None
            prod = [i for i in range(n) if pset.contains([i], [gid])]
            cons = [i for i in range(n) if a["consumer_tiles_per_group"].contains([i], [gid])]
            seed = part if core.core_id in prod else ident
            info.append((prod, cons, seed))
        for core in cores:
            c = core.core_id
            prod, cons, seed = info[c]
            acc = Tile(seed.data.copy(), seed.dtype, seed.data.shape)
            for k in range(1, n):
                o = (c - k) % n
                if o not in prod:
                    continue
                core.push()
                core.set(lhs, acc)
                core.set(rhs, info[o][2])
                r = self.run_ops(core, region.ops)
                core.pop()
                acc = r.values[0] if isinstance(r, _Yield) else r
            if c not in cons:
                # RingReduceBackend returns None off the consumer set and
                # reshape_tile_to_target rejects it (ktdp_helpers.py:186-189)
                raise TypeError("reshape_tile_to_target: expected Tile, got NoneType")
            if not op.results:
                continue
            shape = a.get("result_shape")
            if shape is not None and tuple(shape) != acc.data.shape:
                acc = Tile(acc.data.reshape(shape), acc.dtype, tuple(shape))
            core.set(op.results[0], acc)
            core.track(op.results[0], acc.nbytes())

    # -- grid ------------------------------------------------------------------
    def op_ktdp_get_compute_tile_id(self, core, op):
        if len(op.results) <= 1:
            return core.pos[0]
        return tuple(core.pos[d] for d in range(len(op.results)))

    # -- views and access tiles --------------------------------------------------
    def op_ktdp_construct_memory_view(self, core, op):
        a = op.attributes
        ptr = core.get(op.operands[0])
        shape = tuple(core.get(s) if isinstance(s, str) else s for s in a["shape"])
        strides = [core.get(s) if isinstance(s, str) else s for s in a["strides"]]
        cset = a.get("coordinate_set")
        if isinstance(cset, BoxSet) and not cset.is_concrete:
            syms = tuple(core.get(s) for s in a["shape"] if isinstance(s, str))
            cset = cset.specialize(syms)
        if a["memory_space"] != "HBM":
            raise NotImplementedError("memory views in LX are not supported")
        return MemRef(int(ptr), tuple(int(s) for s in shape), [int(s) for s in strides],
                      a["memory_space"], a["dtype"], cset)

    def op_ktdp_construct_distributed_memory_view(self, core, op):
        """ktir_cpu/dialects/ktdp_ops.py:96-121 with the partition checks of
        DistributedMemRef (ktir_cpu/ir_types.py:140-152)."""
        parts = [core.get(o) for o in op.operands]
        for i, p in enumerate(parts):
            if not isinstance(p, MemRef):
                raise ValueError(f"construct_distributed_memory_view: operand {i} "
                                 f"is {type(p).__name__}, expected MemRef")
        a = op.attributes
        if "shape" not in a or "dtype" not in a:
            raise ValueError("construct_distributed_memory_view: missing required attributes "
                             "'shape'/'dtype'")
        if not parts:
            raise ValueError("DistributedMemRef requires at least one partition")
        for i, p in enumerate(parts):
            if p.coordinate_set is None:
                raise ValueError(f"DistributedMemRef partition {i} must have a coordinate_set")
            if p.dtype != a["dtype"]:
                raise ValueError(f"DistributedMemRef partition {i} dtype {p.dtype!r} "
                                 f"does not match view dtype {a['dtype']!r}")
        return DistRef(parts, tuple(a["shape"]), a["dtype"])

    @staticmethod
    def _dist_route(dist: DistRef, shape, x, acc) -> DistTile:
        """MemoryOps.distributed_tile_access (ktir_cpu/ops/memory_ops.py:651-733):
        per partition C_i = B_i ∩ (x + A); boxes intersect directly, any other
        set is enumerated over the global shape and filtered by membership."""
        nd = len(shape)
        xa = None
        if acc is None:
            xa = (tuple(x), tuple(x[d] + shape[d] for d in range(nd)))
        elif isinstance(acc, BoxSet):
            xa = (tuple(x[d] + acc.lo[d] for d in range(nd)),
                  tuple(x[d] + acc.hi[d] for d in range(nd)))
        out = []
        for part in dist.parts:
            b = part.coordinate_set
            if isinstance(b, BoxSet) and xa is not None:
                lo = tuple(max(b.lo[d], xa[0][d]) for d in range(nd))
                hi = tuple(min(b.hi[d], xa[1][d]) for d in range(nd))
                if any(h <= l for l, h in zip(lo, hi)):
                    continue
                out.append((part, (lo, hi), tuple(b.lo)))
                continue
            pts = b.enumerate_array(tuple(dist.shape))
            if not len(pts):
                continue
            origin = tuple(int(v) for v in pts.min(0))
            keep = np.array([acc.contains(tuple(int(v) for v in p - np.asarray(x)))
                             if acc is not None else
                             all(0 <= p[d] - x[d] < shape[d] for d in range(nd)) for p in pts],
                            bool)
            if keep.any():
                out.append((part, pts[keep], origin))
        if not out:
            raise ValueError(f"distributed_tile_access: no partition covers access region "
                             f"global_base={tuple(x)} shape={tuple(shape)}")
        return DistTile(tuple(x), tuple(shape), out)

    def _dist_refs(self, t: DistTile):
        """Per survivor: (TileRef over the covered points, their coordinates
        inside the access tile, box coordinates or None)."""
        for part, cs, origin in t.survivors:
            nd = len(origin)
            if isinstance(cs, tuple):
                lo, hi = cs
                off = sum((lo[d] - origin[d]) * part.strides[d] for d in range(nd))
                ref = TileRef(part.byte_address + off * bpe(part.dtype),
                              tuple(hi[d] - lo[d] for d in range(nd)), list(part.strides),
                              part.dtype, part.space)
                yield ref, tuple(slice(lo[d] - t.base[d], hi[d] - t.base[d]) for d in range(nd)), None
            else:
                ref = TileRef(part.byte_address, (len(cs),), list(part.strides), part.dtype,
                              part.space)
                local = cs - np.asarray(origin, np.int64)
                yield ref, tuple((cs - np.asarray(t.base, np.int64)).T), local

    def _dist_load(self, t: DistTile, shape, dtype) -> np.ndarray:
        """MemoryOps.distributed_load (ktir_cpu/ops/memory_ops.py:758-846)."""
        out = np.zeros(shape, np_dtype(dtype))
        for ref, at, local in self._dist_refs(t):
            if local is None:
                out[at] = self._load_ref(ref)
            else:
                offs = (local * np.asarray(ref.strides[:local.shape[1]], np.int64)).sum(1)
                out[at] = self.hbm.read_gather(ref.byte, offs, ref.dtype)
        return out

    def _dist_store(self, t: DistTile, data: np.ndarray) -> None:
        """MemoryOps.distributed_store (ktir_cpu/ops/memory_ops.py:848-912)."""
        for ref, at, local in self._dist_refs(t):
            if local is None:
                self._store_ref(ref, np.ascontiguousarray(data[at]))
            else:
                offs = (local * np.asarray(ref.strides[:local.shape[1]], np.int64)).sum(1)
                self.hbm.scatter(ref.byte, offs,
                                 data[at].astype(np_dtype(ref.dtype), copy=False), ref.dtype)

    def op_ktdp_construct_access_tile(self, core, op):
        parent = core.get(op.operands[0])
        idx = [int(core.get(o)) for o in op.operands[1:]]
        a = op.attributes
        if isinstance(parent, DistRef):
            cset = a["coordinate_set"]
            if isinstance(cset, BoxSet) and not cset.is_concrete:
                raise NotImplementedError("construct_access_tile: symbolic access_tile_set")
            return self._dist_route(parent, tuple(a["shape"]),
                                    tuple(int(v) for v in a["base_map"].eval(idx)), cset)
        if not isinstance(parent, MemRef):
            raise TypeError(f"construct_access_tile: parent is {type(parent).__name__}")
        base = a["base_map"].eval(idx)
        off = sum(int(c) * s for c, s in zip(base, parent.strides))
        ref = TileRef(parent.byte_address + off * bpe(parent.dtype), tuple(a["shape"]),
                      list(parent.strides), parent.dtype, parent.space)
        cset = a["coordinate_set"]
        if isinstance(cset, BoxSet) and not cset.is_concrete:
            raise NotImplementedError("construct_access_tile: symbolic access_tile_set")
        return AccessTile(ref, tuple(a["shape"]), cset, a.get("coordinate_order"))

    def op_ktdp_construct_indirect_access_tile(self, core, op):
        a = op.attributes
        parent = core.get(op.operands[0])
        views = [core.get(o) for o in op.operands[1:]]
        consts: Dict[int, int] = {}
        for i, v in enumerate(a["var_names"]):
            if core.has("%" + v):
                val = core.get("%" + v)
                if _is_scalar(val):
                    consts[i] = int(val)
        shape = tuple(a["shape"])
        vss = a["variables_space_set"]
        if consts:
            pts = vss.enumerate_array(shape)
            for i in consts:
                if pts.size and np.any(pts[:, i] != 0):
                    raise ValueError(
                        f"construct_indirect_access_tile: intermediate variable "
                        f"%{a['var_names'][i]} (index {i}) is an outer SSA value but its "
                        f"dimension in variables_space_set has a non-zero range.")
        # resolve outer SSA references inside subscript expressions now
        refs = {}
        for d in a["dims"]:
            for e in (d.get("exprs") or [d.get("expr")]):
                _collect_refs(e, refs)
        for r in list(refs):
            refs[r] = int(core.get(r))
        dims = []
        for d in a["dims"]:
            d2 = dict(d)
            d2["refs"] = refs
            dims.append(d2)
        return IndirectTile(parent, shape, dims, views, vss, a.get("variables_space_order"), consts)

    # -- loads and stores ------------------------------------------------------
    def _load_ref(self, ref: TileRef, coords: Optional[np.ndarray] = None,
                  out_shape=None) -> np.ndarray:
        if coords is None and _contiguous(ref.shape, ref.strides):
            n = int(np.prod(ref.shape))
            return self.hbm.read_bytes(ref.byte, n, ref.dtype).reshape(ref.shape)
        offs = _offsets(ref.shape, ref.strides, coords)
        data = self.hbm.read_gather(ref.byte, offs, ref.dtype)
        return data.reshape(out_shape if out_shape is not None else ref.shape)

    def _store_ref(self, ref: TileRef, data: np.ndarray, coords: Optional[np.ndarray] = None):
        vals = data.astype(np_dtype(ref.dtype), copy=False)
        if coords is None and _contiguous(ref.shape, ref.strides):
            self.hbm.write_bytes(ref.byte, vals.reshape(-1))
            return
        offs = _offsets(ref.shape, ref.strides, coords)
        self.hbm.scatter(ref.byte, offs, vals.reshape(-1), ref.dtype)

    @staticmethod
    def _sub_ref(ref: TileRef, box: BoxSet) -> TileRef:
        off = sum(lo * s for lo, s in zip(box.lo, ref.strides))
        return TileRef(ref.byte + off * bpe(ref.dtype), box.extent(), ref.strides, ref.dtype,
                       ref.space)

    def _coords(self, at: AccessTile) -> np.ndarray:
        pts = at.cset.enumerate_array(at.shape)
        if at.order is not None:
            out = at.order.eval(list(pts.T))
            pts = np.stack([np.broadcast_to(np.asarray(o, np.int64), (pts.shape[0],))
                            for o in out], axis=1)
        return pts

    def op_ktdp_load(self, core, op):
        t = core.get(op.operands[0])
        rshape = op.attributes.get("result_shape")
        if isinstance(t, DistTile):
            dt = t.survivors[0][0].dtype
            data = self._dist_load(t, tuple(rshape or t.shape), dt)
            return Tile(data, dt, tuple(data.shape))
        if isinstance(t, IndirectTile):
            ref, coords = self._indirect_coords(t)
            data = self._load_ref(ref, coords, rshape or t.shape)
            return Tile(data, ref.dtype, tuple(data.shape))
        if isinstance(t.cset, BoxSet) and t.order is None:
            sub = self._sub_ref(t.ref, t.cset)
            data = self._load_ref(sub)
            return Tile(data, sub.dtype, sub.shape)
        coords = self._coords(t)
        data = self._load_ref(t.ref, coords, rshape or t.shape)
        return Tile(data, t.ref.dtype, tuple(data.shape))

    def op_ktdp_store(self, core, op):
        tile = core.get(op.operands[0])
        if not isinstance(tile, Tile):
            raise TypeError(f"ktdp.store expects a Tile, got {type(tile)}")
        t = core.get(op.operands[1])
        if isinstance(t, DistTile):
            self._dist_store(t, tile.data)
            return None
        if isinstance(t, IndirectTile):
            if tuple(tile.shape) != tuple(t.shape):
                raise ValueError(
                    f"indirect_store: source tile shape {tuple(tile.shape)} does not match "
                    f"IAT shape {tuple(t.shape)}")
            ref, coords = self._indirect_coords(t)
            self._store_ref(ref, tile.data, coords)
            return None
        if isinstance(t.cset, BoxSet) and t.order is None:
            self._store_ref(self._sub_ref(t.ref, t.cset), tile.data)
            return None
        self._store_ref(t.ref, tile.data, self._coords(t))
        return None

    def _indirect_coords(self, t: IndirectTile):
        if t.vso is not None and not t.vso.is_permutation():
            raise ValueError("indirect access: variables_space_order must permute its input "
                             f"dimensions; got non-permutation map: {t.vso.source}")
        pts = t.vss.enumerate_array(t.shape)
        if t.vso is not None and len(pts):
            keys = np.stack([np.broadcast_to(np.asarray(k, np.int64), (pts.shape[0],))
                             for k in t.vso.eval(list(pts.T))], axis=1)
            order = np.lexsort(keys.T[::-1])
            pts = pts[order]
        for i, v in t.consts.items():
            pts = pts.copy()
        cols = list(pts.T) if len(pts) else [np.zeros(0, np.int64)] * pts.shape[1]
        coords = []
        for d in t.dims:
            refs = d["refs"]
            if d["kind"] == "direct":
                e = d["expr"]
                vals = _eval_dim(e, cols, t.consts, refs, pts.shape[0])
                coords.append(vals)
            else:
                view = t.views[d["view"]]
                off = np.zeros(pts.shape[0], np.int64)
                for e, s in zip(d["exprs"], view.strides):
                    off = off + _eval_dim(e, cols, t.consts, refs, pts.shape[0]) * s
                idx = self._read_index(view, off)
                if idx.size and idx.min() < 0:
                    bad = int(idx[idx < 0][0])
                    raise IndexError(f"indirect index {bad} from {view} is negative")
                coords.append(idx.astype(np.int64))
        coords_arr = np.stack(coords, axis=1) if coords else np.zeros((0, 0), np.int64)
        pr = t.parent
        ref = TileRef(pr.byte_address, pr.shape, pr.strides, pr.dtype, pr.space)
        return ref, coords_arr

    def _read_index(self, view: MemRef, off: np.ndarray) -> np.ndarray:
        if off.size == 0:
            return np.zeros(0, np.int64)
        # read_scattered: runs of adjacent addresses are read from the
        # allocation holding the run's first address (zero past its end).
        uniq = np.unique(off)
        starts = np.concatenate([[True], np.diff(uniq) != 1])
        run_id = np.cumsum(starts) - 1
        run_start = uniq[starts]
        vals = np.zeros(uniq.size, dtype=np.int64)
        for r, s in enumerate(run_start):
            sel = run_id == r
            n = int(sel.sum())
            block = self.hbm.read_bytes(view.byte_address + int(s) * bpe(view.dtype), n, view.dtype)
            vals[sel] = block
        pos = np.searchsorted(uniq, off)
        return vals[pos]

    # -- constants, casts, elementwise ------------------------------------------
    def op_arith_constant(self, core, op):
        a = op.attributes
        if a.get("is_tensor"):
            dt = np_dtype(a["dtype"])
            if a.get("dense_list"):
                return Tile(np.array(a["value"], dtype=dt).reshape(a["shape"]), a["dtype"],
                            tuple(a["shape"]))
            return Tile(np.full(a["shape"], a["value"], dtype=dt), a["dtype"], tuple(a["shape"]))
        return a.get("value", 0)

    def _elementwise_handler(self, name):
        fb = _FLOAT_BIN.get(name)
        if fb is not None:
            return lambda core, op: _float_binop(core, op, fb)
        ib = _INT_BIN.get(name)
        if ib is not None:
            return lambda core, op: _int_binop(core, op, ib)
        mu = _MATH_UNARY.get(name)
        if mu is not None:
            return lambda core, op: _math_unary(core, op, mu)
        return None

    def op_arith_maxnumf(self, core, op):
        return _minmax(core, op, np.fmax)

    def op_arith_minnumf(self, core, op):
        return _minmax(core, op, np.fmin)

    def op_arith_maximumf(self, core, op):
        return _minmax(core, op, np.maximum)

    op_arith_maxf = op_arith_maximumf

    def op_arith_minimumf(self, core, op):
        return _minmax(core, op, np.minimum)

    op_arith_minf = op_arith_minimumf

    def op_arith_maxsi(self, core, op):
        return _minmax(core, op, np.maximum, scalar=max)

    def op_arith_minsi(self, core, op):
        return _minmax(core, op, np.minimum, scalar=min)

    op_arith_maxui = op_arith_maxsi
    op_arith_minui = op_arith_minsi

    def op_arith_negf(self, core, op):
        v = core.get(op.operands[0])
        return Tile(-v.data, v.dtype, v.shape) if isinstance(v, Tile) else -v

    def op_arith_absf(self, core, op):
        v = core.get(op.operands[0])
        return Tile(np.abs(v.data), v.dtype, v.shape) if isinstance(v, Tile) else abs(v)

    op_math_absf = op_arith_absf
    op_math_absi = op_arith_absf

    def op_arith_cmpi(self, core, op):
        return _cmp(core, op, integer=True)

    def op_arith_cmpf(self, core, op):
        return _cmp(core, op, integer=False)

    def op_arith_select(self, core, op):
        c = core.get(op.operands[0])
        t = core.get(op.operands[1])
        f = core.get(op.operands[2])
        if isinstance(c, (Tile, np.ndarray)):
            cd = c.data if isinstance(c, Tile) else c
            td = t.data if isinstance(t, Tile) else t
            fd = f.data if isinstance(f, Tile) else f
            r = np.where(cd, td, fd)
            ref = t if isinstance(t, Tile) else f
            dt = ref.dtype if isinstance(ref, Tile) else "f16"
            shape = ref.shape if isinstance(ref, Tile) else r.shape
            return Tile(r, dt, shape)
        return t if c else f

    def _cast(self, core, op, target, floating: bool, opname: str):
        v = core.get(op.operands[0])
        label = KTIR_OF.get(np.dtype(target))
        if isinstance(v, Tile):
            if v.data.dtype == target:
                return v
            cat = np.floating if floating else np.integer
            if not np.issubdtype(v.data.dtype, cat):
                raise TypeError(f"{opname} expects {'float' if floating else 'integer'} Tile")
            return Tile(v.data.astype(target), label, v.shape)
        if isinstance(v, target):
            return v
        r = target(v)
        if np.issubdtype(np.dtype(target), np.floating) and np.isinf(r) and not np.isinf(float(v)):
            raise OverflowError(f"{opname}: {v} overflows {target.__name__}")
        return r

    def op_arith_extf(self, core, op):
        v = core.get(op.operands[0])
        if not isinstance(v, Tile):
            return np.float32(v)
        return self._cast(core, op, np.float32, True, "extf")

    def op_arith_convertf(self, core, op):
        # ktir_cpu/ops/arith_ops.py:660-668
        v = core.get(op.operands[0])
        if isinstance(v, Tile):
            if v.data.dtype == np.float16:
                return Tile(v.data.astype(np.float32), "f32", v.shape)
            return Tile(v.data.astype(np.float16), "f16", v.shape)
        return np.float32(v) if isinstance(v, np.float16) else np.float16(v)

    def op_ktdp_coreid(self, core, op):
        # ktir_cpu/ops/grid_ops.py:43-62 with ktir_cpu/grid.py:402-470
        want = ([int(core.get(o)) for o in op.operands] + [0, 0, 0])[:3]
        nx, ny, nz = self.grid
        out = []
        for cid in range(nx * ny * nz):
            z, r = divmod(cid, nx * ny)
            y, x = divmod(r, nx)
            if all(w == -1 or w == p for w, p in zip(want, (x, y, z))):
                out.append(cid)
        return out

    def op_arith_truncf(self, core, op):
        return self._cast(core, op, np.float16, True, "truncf")

    def op_arith_sitofp(self, core, op):
        v = core.get(op.operands[0])
        dst = op.attributes.get("dst_type") or (op.result_types[0] if op.result_types else "f32")
        dname = _elem(dst) or "f32"
        dt = np_dtype(dname)
        if isinstance(v, Tile):
            return Tile(v.data.astype(dt), dname, v.shape)
        return np.dtype(dt).type(v)

    def op_arith_uitofp(self, core, op):
        v = core.get(op.operands[0])
        if isinstance(v, Tile):
            return Tile(v.data.astype(np.float32), "f32", v.shape)
        return float(v)

    def op_arith_fptosi(self, core, op):
        v = core.get(op.operands[0])
        if isinstance(v, Tile):
            return Tile(v.data.astype(np.int32), "i32", v.shape)
        return int(v)

    def op_arith_fptoui(self, core, op):
        # ops/arith_ops.py:504-508: a uint32 tile labelled "ui32"
        v = core.get(op.operands[0])
        if isinstance(v, Tile):
            return Tile(v.data.astype(np.uint32), "ui32", v.shape)
        return int(v)

    def op_arith_extsi(self, core, op):
        v = core.get(op.operands[0])
        if isinstance(v, Tile):
            return Tile(v.data.astype(np.int64), "i64", v.shape)
        return int(v)

    op_arith_extui = op_arith_extsi

    def op_arith_trunci(self, core, op):
        v = core.get(op.operands[0])
        if isinstance(v, Tile):
            return Tile(v.data.astype(np.int32), "i32", v.shape)
        return int(v)

    def op_arith_index_cast(self, core, op):
        return int(core.get(op.operands[0]))

    op_arith_index_castui = op_arith_index_cast

    def op_arith_bitcast(self, core, op):
        v = core.get(op.operands[0])
        dst = _elem(op.attributes.get("dst_type", "f32")) or "f32"
        if isinstance(v, Tile):
            return Tile(v.data.view(np_dtype(dst)), dst, v.shape)
        if dst == "f32":
            return float(np.frombuffer(int(v).to_bytes(4, "little", signed=(v < 0)),
                                       dtype=np.float32)[0])
        return int(np.frombuffer(np.float32(v).tobytes(), dtype=np.int32)[0])

    def op_math_fma(self, core, op):
        a, b, c = (core.get(o) for o in op.operands[:3])
        if isinstance(a, Tile):
            r = (a.data.astype(np.float32) * b.data.astype(np.float32) +
                 c.data.astype(np.float32)).astype(a.data.dtype)
            return Tile(r, a.dtype, a.shape)
        return type(a)(float(a) * float(b) + float(c))

    def op_math_powf(self, core, op):
        a, b = (core.get(o) for o in op.operands[:2])
        if isinstance(a, Tile):
            bd = b.data if isinstance(b, Tile) else np.float32(b)
            r = np.power(a.data.astype(np.float32), np.asarray(bd).astype(np.float32))
            return Tile(r.astype(a.data.dtype), a.dtype, a.shape)
        return type(a)(float(a) ** float(b))

    # -- tensor dialect ----------------------------------------------------------
    def op_tensor_empty(self, core, op):
        a = op.attributes
        return Tile(np.zeros(a["shape"], dtype=np_dtype(a["dtype"])), a["dtype"], tuple(a["shape"]))

    def op_tensor_splat(self, core, op):
        s = core.get(op.operands[0])
        if isinstance(s, Tile):
            s = s.data.flat[0]
        shape = tuple(op.attributes.get("shape", ()))
        dt = op.attributes.get("dtype", "f16")
        if not shape:
            shape = (1,)
        if isinstance(s, (np.integer, int)) and not isinstance(s, (bool, np.bool_)):
            return Tile(np.full(shape, s, dtype=np.int32), "i32", shape)
        return Tile(np.full(shape, s, dtype=np_dtype(dt)), dt, shape)

    def op_tensor_extract(self, core, op):
        src = core.get(op.operands[0])
        if isinstance(src, Tile):
            idx = [int(core.get(o)) for o in op.operands[1:]]
            if not idx:
                return src.data.flat[0]
            return src.data[tuple(idx)]
        return src

    def _reshape(self, core, op):
        src = core.get(op.operands[0])
        ts = op.attributes.get("target_shape")
        if isinstance(src, Tile) and ts:
            return Tile(src.data.reshape(ts), src.dtype, tuple(ts))
        return src

    op_tensor_expand_shape = _reshape
    op_tensor_collapse_shape = _reshape
    op_tensor_reshape = _reshape

    def op_tensor_from_elements(self, core, op):
        vals = []
        for o in op.operands:
            v = core.get(o)
            vals.append(v.data.flat[0] if isinstance(v, Tile) else v)
        a = op.attributes
        return Tile(np.array(vals, dtype=np_dtype(a["dtype"])).reshape(a["shape"]), a["dtype"],
                    tuple(a["shape"]))

    def op_tensor_generate(self, core, op):
        a = op.attributes
        shape = tuple(a["shape"])
        region = op.regions[0]
        grids = np.meshgrid(*(np.arange(s) for s in shape), indexing="ij")
        core.push()
        for (name, _), g in zip(region.args, grids):
            core.set(name, Tile(g, "index", shape))
        r = self.run_region(core, region)
        if isinstance(r, _Yield):
            r = r.values[0]
        core.pop()
        dt = np_dtype(a["dtype"])
        data = r.data.astype(dt) if isinstance(r, Tile) else np.full(shape, r, dtype=dt)
        return Tile(data, a["dtype"], shape)

    def op_tensor_yield(self, core, op):
        return _Yield([core.get(o) for o in op.operands])

    op_linalg_yield = op_tensor_yield
    op_scf_yield = op_tensor_yield

    def op_return(self, core, op):
        return core.get(op.operands[0]) if op.operands else None

    # -- linalg ----------------------------------------------------------------
    def _combine(self, core, region_args, body, lhs, rhs):
        core.push()
        if region_args:
            core.set(region_args[0], lhs)
        if len(region_args) > 1:
            core.set(region_args[1], rhs)
        r = self.run_ops(core, body)
        core.pop()
        return r.values[0] if isinstance(r, _Yield) else r

    def op_linalg_reduce(self, core, op):
        t = core.get(op.operands[0])
        a = op.attributes
        if op.regions and op.regions[0].ops:
            region = op.regions[0]
            names = linalg_block_args(region)
            body = region.ops
        else:
            comb = a.get("combiner") or "arith.addf"
            names = ["%__in", "%__acc"]
            body = [Operation(comb, ["%__r"], names, {}, []),
                    Operation("linalg.yield", [], ["%__r"], {}, [])]
        dims = a.get("dims")
        dim = dims[0] if dims else None
        if not isinstance(t, Tile):
            res = t
        else:
            data = t.data
            if dim is None:
                data = data.reshape(-1)
                dim = 0
            acc = data
            n = acc.shape[dim]
            while n > 1:
                h = n // 2
                left = np.take(acc, np.arange(0, h), axis=dim)
                right = np.take(acc, np.arange(h, 2 * h), axis=dim)
                c = self._combine(core, names, body, Tile(left, t.dtype, left.shape),
                                  Tile(right, t.dtype, right.shape))
                c = c.data if isinstance(c, Tile) else np.asarray(c)
                if n % 2:
                    c = np.concatenate([c, np.take(acc, np.arange(2 * h, n), axis=dim)], axis=dim)
                acc = c
                n = acc.shape[dim]
            if dims is None:
                res = acc.reshape(()).astype(t.data.dtype).item()
            else:
                red = np.squeeze(acc, axis=dim).astype(t.data.dtype)
                res = red.item() if red.ndim == 0 else Tile(red, t.dtype, red.shape)
        outs = a.get("outs")
        if outs and res is not None:
            core.set(outs, res)
        return res

    def op_linalg_add(self, core, op):
        x = core.get(op.operands[0])
        y = core.get(op.operands[1])
        return Tile(x.data + y.data, x.dtype, x.shape)

    def op_linalg_fill(self, core, op):
        s = core.get(op.operands[0])
        o = core.get(op.operands[1])
        return Tile(np.full(o.shape, float(s), dtype=o.data.dtype), o.dtype, o.shape)

    def op_linalg_broadcast(self, core, op):
        x = core.get(op.operands[0])
        o = core.get(op.operands[1])
        data = x.data
        for d in sorted(op.attributes.get("dimensions", [])):
            data = np.expand_dims(data, axis=d)
        return Tile(np.broadcast_to(data, o.shape).copy(), x.dtype, tuple(o.shape))

    def op_linalg_matmul(self, core, op):
        x = core.get(op.operands[0])
        y = core.get(op.operands[1])
        r = np.matmul(x.data, y.data).astype(x.data.dtype)
        res = Tile(r, x.dtype, (x.shape[0], y.shape[1]))
        if len(op.operands) > 2:
            acc = core.get(op.operands[2])
            if isinstance(acc, Tile):
                res = Tile(acc.data + res.data, acc.dtype, acc.shape)
        return res

    def op_linalg_batch_matmul(self, core, op):
        x = core.get(op.operands[0])
        y = core.get(op.operands[1])
        p = x.data @ y.data
        res = Tile(p, x.dtype, p.shape)
        if len(op.operands) > 2:
            acc = core.get(op.operands[2])
            if isinstance(acc, Tile):
                res = Tile(acc.data + res.data, acc.dtype, acc.shape)
        return res

    def op_linalg_transpose(self, core, op):
        x = core.get(op.operands[0])
        perm = op.attributes["permutation"]
        return Tile(np.transpose(x.data, perm).copy(), x.dtype, tuple(x.shape[i] for i in perm))

    def op_linalg_generic(self, core, op):
        a = op.attributes
        n_ins = a["n_ins"]
        maps = a["indexing_maps"]
        ins = [core.get(o) for o in op.operands[:n_ins]]
        outs = core.get(op.operands[n_ins])
        region = op.regions[0]
        names = linalg_block_args(region)
        shape = outs.shape
        core.push()
        core.set("__linalg_shape__", shape)
        for i, (v, m) in enumerate(zip(ins, maps[:n_ins])):
            dims = [e[1] for e in m.exprs if e[0] == "d"]
            if isinstance(v, Tile):
                data = v.data
                for d in range(len(shape)):
                    if d not in dims:
                        data = np.expand_dims(data, axis=d)
                arg = Tile(np.broadcast_to(data, shape).copy(), v.dtype, shape)
            else:
                arg = v
            if i < len(names):
                core.set(names[i], arg)
        if n_ins < len(names):
            core.set(names[n_ins], Tile(outs.data.copy(), outs.dtype, shape))
        r = self.run_ops(core, region.ops)
        core.pop()
        if isinstance(r, _Yield):
            r = r.values[0] if len(r.values) == 1 else tuple(r.values)
        dt = outs.data.dtype
        if isinstance(r, Tile):
            return Tile(np.broadcast_to(r.data, shape).copy().astype(dt), outs.dtype, shape)
        return Tile(np.full(shape, r, dtype=dt), outs.dtype, shape)

    def op_linalg_index(self, core, op):
        d = op.attributes["dim"]
        shape = core.get("__linalg_shape__")
        idx = np.arange(shape[d], dtype=np.int64)
        rs = [1] * len(shape)
        rs[d] = shape[d]
        return Tile(idx.reshape(rs), "index", tuple(rs))

    # -- control flow ---------------------------------------------------------------
    def op_scf_for(self, core, op):
        lb, ub, st = (int(core.get(o)) for o in op.operands[:3])
        names = op.attributes.get("iter_args", [])
        cur = [core.get(o) for o in op.operands[3:]]
        for name, v in zip(names, cur):
            core.set(name, v)
            if isinstance(v, Tile):
                core.track(name, v.nbytes())
        body = op.regions[0]
        iv = op.attributes["iter_var"]
        its = range(lb, ub, max(st, 1))
        if self.loop_limit is not None and self._for_depth == 0 and len(its) > self.loop_limit:
            self.loop_fraction = self.loop_limit / len(its)
            its = its[:self.loop_limit]
        self._for_depth += 1
        try:
            return self._for_iterations(core, op, its, body, iv, names, cur)
        finally:
            self._for_depth -= 1

    def _for_iterations(self, core, op, its, body, iv, names, cur):
        for i in its:
            core.push()
            core.set(iv, i)
            r = self.run_region(core, body)
            ys = r.values if isinstance(r, _Yield) and names else None
            core.pop()
            if ys is not None:
                for name, v in zip(names, ys):
                    core.untrack(name)
                    core.set(name, v)
                    if isinstance(v, Tile):
                        core.track(name, v.nbytes())
                cur = list(ys)
        if not cur:
            return None
        return cur[0] if len(cur) == 1 else tuple(cur)

    def op_scf_if(self, core, op):
        c = core.get(op.operands[0])
        region = op.regions[0] if c else (op.regions[1] if len(op.regions) > 1 else None)
        if region is None or not region.ops:
            return None
        core.push()
        r = self.run_region(core, region)
        core.pop()
        if isinstance(r, _Yield):
            if not r.values:
                return None
            return r.values[0] if len(r.values) == 1 else tuple(r.values)
        return r


# ---------------------------------------------------------------------------
# elementwise helpers
# ---------------------------------------------------------------------------

def _elem(t: Optional[str]) -> Optional[str]:
    if not t:
        return None
    t = t.strip()
    if t.startswith("tensor<"):
        inner = t[len("tensor<"):-1]
        return inner.split("x")[-1]
    return t


def _float_binop(core, op, fn):
    a = core.get(op.operands[0])
    b = core.get(op.operands[1])
    if _is_scalar(a) and _is_scalar(b):
        r = fn(np.float16(a), np.float16(b))
        return r if isinstance(r, np.float16) else np.float16(r)
    if isinstance(a, Tile) and isinstance(b, Tile):
        return Tile(fn(a.data, b.data), a.dtype, a.shape)
    if isinstance(a, Tile):
        return Tile(fn(a.data, np.float16(b)), a.dtype, a.shape)
    return Tile(fn(np.float16(a), b.data), b.dtype, b.shape)


def _int_binop(core, op, fn):
    a = core.get(op.operands[0])
    b = core.get(op.operands[1])
    if isinstance(a, Tile) or isinstance(b, Tile):
        if isinstance(a, Tile) and isinstance(b, Tile):
            return Tile(fn(a.data, b.data), a.dtype, a.shape)
        if isinstance(a, Tile):
            return Tile(fn(a.data, int(b)), a.dtype, a.shape)
        return Tile(fn(int(a), b.data), b.dtype, b.shape)
    return fn(a, b)


def _truncdiv(a, b):
    return np.trunc(a / b).astype(np.asarray(a).dtype) if isinstance(a, np.ndarray) or \
        isinstance(b, np.ndarray) else int(np.trunc(a / b))


def _truncrem(a, b):
    return np.asarray(a) - _truncdiv(a, b) * np.asarray(b) if isinstance(a, np.ndarray) or \
        isinstance(b, np.ndarray) else a - _truncdiv(a, b) * b


def _ceildiv(a, b):
    if isinstance(a, np.ndarray) or isinstance(b, np.ndarray):
        dt = (a if isinstance(a, np.ndarray) else b).dtype
        return np.ceil(a / b).astype(dt)
    return math.ceil(a / b)


def _shrui(a, b):
    if isinstance(a, np.ndarray):
        return (a.astype(np.uint64) >> np.uint64(b)).astype(a.dtype)
    return (a & 0xFFFFFFFFFFFFFFFF) >> b


_FLOAT_BIN = {
    "arith.addf": operator.add, "arith.subf": operator.sub, "arith.mulf": operator.mul,
    "arith.divf": operator.truediv, "arith.remf": operator.mod,
}
_INT_BIN = {
    "arith.addi": operator.add, "arith.subi": operator.sub, "arith.muli": operator.mul,
    "arith.divui": operator.floordiv, "arith.divsi": _truncdiv, "arith.floordivsi": operator.floordiv,
    "arith.remui": operator.mod, "arith.remsi": _truncrem, "arith.ceildivsi": _ceildiv,
    "arith.ceildivui": _ceildiv, "arith.andi": operator.and_, "arith.ori": operator.or_,
    "arith.xori": operator.xor, "arith.shli": operator.lshift, "arith.shrsi": operator.rshift,
    "arith.shrui": _shrui,
}


def _erf32(x):
    a = np.abs(x)
    t = 1.0 / (1.0 + 0.3275911 * a)
    poly = t * (0.254829592 + t * (-0.284496736 + t * (1.421413741 + t * (-1.453152027 + t * 1.061405429))))
    return np.sign(x) * (1.0 - poly * np.exp(-a * a))


_MATH_UNARY = {
    "math.exp": np.exp, "math.sqrt": np.sqrt, "math.rsqrt": lambda x: 1.0 / np.sqrt(x),
    "math.log": np.log, "math.log2": np.log2, "math.log1p": np.log1p, "math.tanh": np.tanh,
    "math.sin": np.sin, "math.cos": np.cos, "math.ceil": np.ceil, "math.floor": np.floor,
    "math.erf": _erf32,
}


def _math_unary(core, op, fn):
    v = core.get(op.operands[0])
    if isinstance(v, Tile):
        r = fn(v.data.astype(np.float32)).astype(v.data.dtype)
        return Tile(r, v.dtype, v.shape)
    if op.op_type == "math.erf":
        return type(v)(_erf32(np.array([float(v)]))[0])
    return type(v)(fn(float(v)))


def _minmax(core, op, fn, scalar=None):
    a = core.get(op.operands[0])
    b = core.get(op.operands[1])
    if isinstance(a, Tile) or isinstance(b, Tile):
        ad = a.data if isinstance(a, Tile) else a
        bd = b.data if isinstance(b, Tile) else b
        ref = a if isinstance(a, Tile) else b
        return Tile(fn(ad, bd), ref.dtype, ref.shape)
    if scalar is not None:
        return scalar(a, b)
    return fn(a, b)


def _cmp(core, op, integer: bool):
    a = core.get(op.operands[0])
    b = core.get(op.operands[1])
    pred = op.attributes["predicate"]
    is_tile = isinstance(a, Tile) or isinstance(b, Tile)
    if is_tile:
        lhs = a.data if isinstance(a, Tile) else np.full(b.shape, a, dtype=b.data.dtype)
        rhs = b.data if isinstance(b, Tile) else np.full(a.shape, b, dtype=a.data.dtype)
    elif integer:
        lhs, rhs = a, b
    else:
        lhs, rhs = float(a), float(b)
    nan = (lambda: np.isnan(lhs) | np.isnan(rhs))
    table = {
        "eq": lambda: lhs == rhs, "ne": lambda: lhs != rhs,
        "slt": lambda: lhs < rhs, "ult": lambda: lhs < rhs, "sle": lambda: lhs <= rhs,
        "ule": lambda: lhs <= rhs, "sgt": lambda: lhs > rhs, "ugt": lambda: lhs > rhs,
        "sge": lambda: lhs >= rhs, "uge": lambda: lhs >= rhs,
    } if integer else {
        "false": lambda: np.zeros_like(lhs, dtype=bool) if is_tile else False,
        "true": lambda: np.ones_like(lhs, dtype=bool) if is_tile else True,
        "oeq": lambda: lhs == rhs, "olt": lambda: lhs < rhs, "ole": lambda: lhs <= rhs,
        "ogt": lambda: lhs > rhs, "oge": lambda: lhs >= rhs,
        "one": lambda: (lhs != rhs) & ~nan(),
        "ueq": lambda: (lhs == rhs) | nan(), "une": lambda: lhs != rhs,
        "ult": lambda: (lhs < rhs) | nan(), "ule": lambda: (lhs <= rhs) | nan(),
        "ugt": lambda: (lhs > rhs) | nan(), "uge": lambda: (lhs >= rhs) | nan(),
        "ord": lambda: ~nan(), "uno": lambda: nan(),
    }
    if pred not in table:
        raise NotImplementedError(f"{op.op_type}: unsupported predicate '{pred}'")
    r = table[pred]()
    if is_tile:
        r = np.asarray(r)
        return Tile(r, "i1", r.shape)
    return bool(r) if not isinstance(r, bool) else r


def _collect_refs(e, out: dict):
    if e is None:
        return
    if e[0] == "ref":
        out[e[1]] = None
        return
    for c in e[1:]:
        if isinstance(c, tuple):
            _collect_refs(c, out)


def _eval_dim(expr, cols, consts, refs, n):
    # intermediate variables bound to an outer SSA scalar evaluate to that value
    cols2 = list(cols)
    for i, v in consts.items():
        cols2[i] = np.full(n, v, dtype=np.int64)
    v = eval_expr(expr, cols2, (), refs)
    return np.broadcast_to(np.asarray(v, dtype=np.int64), (n,))
