"""KTIRInterpreter: the reference's Python API, executing on a B200.

Same surface as ktir_cpu/interpreter.py:38-316 — ``load``,
``execute_function``, ``arg_names``, ``tensor_input_output_sizes``,
``get_latency_report``, the ``_prepare_execution(grid_shape)`` hook and the
``memory.hbm`` read/write façade that tests use to seed memory at fixed stick
addresses — with execution redirected: the function is traced once per call
signature (pointer layout, scalar values, tensor shapes), lowered to device
programs, and replayed on the GPU for every call with that signature.

Error behaviour follows the reference: ``RuntimeError("No module loaded...")``,
``ValueError`` for unknown ops / unmapped reads, ``MemoryError`` on LX
overflow, ``IndexError`` for a negative indirect index (reported by the
device and raised after the call), ``NotImplementedError`` for programs whose
schedule depends on tile data.
"""

from __future__ import annotations

import ctypes as C
import os
import sys
from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from . import runtime as R
from .ir import IRModule
from .lower import Lowerer, Plan
from .parser import KTIRParser, KTIRParserBase
from .trace import STICK, AddressSpace, Tracer

_KTIR_OF = {np.dtype(np.float16): "f16", np.dtype(np.float32): "f32",
            np.dtype(np.int32): "i32", np.dtype(np.int64): "i64"}


class HBMFacade:
    """Host view of the simulated HBM: stick-addressed allocations.

    Mirrors HBMSimulator.allocate/read/write (ktir_cpu/memory.py:201-288) so
    callers can seed and inspect memory around a call.  Data lives here on
    the host between calls; each call uploads it, runs, and reads it back.
    """

    STICK_BYTES = STICK

    def __init__(self) -> None:
        self.allocs: Dict[int, np.ndarray] = {}     # byte address -> flat array
        self.borrowed: set = set()                  # allocations aliasing caller arrays
        self.next_ptr = 0x10000

    def allocate(self, size: int) -> int:
        ptr = self.next_ptr
        self.next_ptr = (ptr + size + STICK - 1) & ~(STICK - 1)
        return ptr // STICK

    def _find(self, addr: int):
        if addr in self.allocs:
            return addr, self.allocs[addr]
        for base, arr in self.allocs.items():
            if base < addr < base + arr.nbytes:
                return base, arr
        return None

    def attach(self, stick: int, data: np.ndarray) -> None:
        """Make `data` the allocation at `stick` without copying it; the façade
        copies it first if it is ever written through `write`."""
        addr = stick * STICK
        self.allocs[addr] = np.ascontiguousarray(data).reshape(-1)
        self.borrowed.add(addr)

    def write(self, stick: int, data: np.ndarray, *, intra_byte: int = 0) -> None:
        addr = stick * STICK + intra_byte
        flat = np.ascontiguousarray(data).reshape(-1)
        found = self._find(addr)
        if found is None:
            self.allocs[addr] = flat.copy()
            return
        base, arr = found
        if base in self.borrowed:
            arr = self.allocs[base] = arr.copy()
            self.borrowed.discard(base)
        off = (addr - base) // flat.itemsize
        fit = max(0, min(flat.size, arr.size - off))
        arr[off:off + fit] = flat[:fit]

    def read(self, stick: int, n_elements: int, dtype: str, *, intra_byte: int = 0) -> np.ndarray:
        from .trace import np_dtype
        addr = stick * STICK + intra_byte
        found = self._find(addr)
        if found is None:
            raise ValueError(f"Read from unmapped address 0x{addr:x} (n_elements={n_elements})")
        base, arr = found
        dt = np_dtype(dtype)
        off = (addr - base) // dt.itemsize
        out = np.zeros(n_elements, dtype=dt)
        avail = max(0, min(n_elements, arr.size - off))
        out[:avail] = arr[off:off + avail]
        return out


class LXFacade(HBMFacade):
    """Host view of one core's LX scratchpad: byte-addressed allocations, read
    and written like ktir_cpu/memory.py:304-331 (reads past an allocation
    return zeros, writes are truncated), so tests can seed it before a call."""

    def write(self, ptr: int, data: np.ndarray) -> None:  # type: ignore[override]
        super().write(0, data, intra_byte=ptr)

    def read(self, ptr: int, n_elements: int, dtype: str) -> np.ndarray:  # type: ignore[override]
        return super().read(0, n_elements, dtype, intra_byte=ptr)


class DeviceMemory:
    """The interpreter's `memory` attribute: the HBM façade and per-core LX
    scratchpads (`get_lx(core)`).  Every allocation of either becomes one
    device buffer of a call; LX allocations live in the address space at
    `lx_address(core, byte)`, apart from HBM."""

    def __init__(self, num_cores: int) -> None:
        self.num_cores = num_cores
        self.hbm = HBMFacade()
        self.lx: Dict[int, LXFacade] = {}

    def get_lx(self, core_id: int) -> LXFacade:
        if core_id < 0 or core_id >= self.num_cores:
            raise ValueError(f"core {core_id} is out of range [0, {self.num_cores})")
        return self.lx.setdefault(core_id, LXFacade())

    def allocations(self) -> List[Tuple[int, Any, int]]:
        """(address in the trace's address space, façade, façade key), sorted."""
        from .trace import lx_address
        out = [(a, self.hbm, a) for a in self.hbm.allocs]
        for core, lx in self.lx.items():
            out += [(lx_address(core, a), lx, a) for a in lx.allocs]
        return sorted(out, key=lambda t: t[0])


class Executable:
    """A traced + lowered call signature, replayable on device buffers."""

    def __init__(self, plan: Plan, space: AddressSpace, device, grid):
        import torch
        self.torch = torch
        self.plan = plan
        self.space = space
        self.device = device
        self.grid = grid
        self.lib = R.load_library()
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.dev_tensors = None
        self.latency_tape = None
        self.pinned = None
        self.status_pinned = None
        self.last_h2d_bytes = self.last_d2h_bytes = 0
        self.bufs = None
        self.arena = None
        if plan.arena_bytes:
            self.arena = torch.zeros(plan.arena_bytes + 256, dtype=torch.uint8, device=device)
            for byte_off, arr in plan.info.get("dense_uploads", []):
                src = torch.from_numpy(arr.view(np.uint8).reshape(-1).copy())
                self.arena[byte_off:byte_off + src.numel()].copy_(src)

    def buffers(self, tensors: List[Any]) -> R.KtirBuffers:
        b = R.KtirBuffers()
        for i, t in enumerate(tensors):
            b.base[i] = t.data_ptr()
            b.numel[i] = self.space.buffers[i].numel
        if self.arena is not None:
            b.base[R.ARENA_SLOT] = self.arena.data_ptr()
            b.numel[R.ARENA_SLOT] = 1 << 62
        return b

    def launch(self, tensors: List[Any], stream=None, bufs: Optional[R.KtirBuffers] = None) -> None:
        """Enqueue the plan on `stream` over device tensors (one per buffer, in address order)."""
        s = stream if stream is not None else self.torch.cuda.current_stream(self.device)
        sp = C.c_void_p(s.cuda_stream)
        if bufs is None:
            bufs = self.buffers(tensors)
        st = self.status.data_ptr()
        for l in self.plan.launches:
            l.fn(bufs, sp, st)

    def capture(self, tensor_sets: List[List[Any]], stream=None):
        """Record the plan once per tensor set, in order, into one CUDA graph.

        Replaying the graph runs exactly those executions with a single host
        launch, for callers that issue many executions back to back (the
        per-execution host cost of `launch` is then paid once).  Every launch of
        the plan must already have run once outside capture (one-time kernel
        attribute setup).  Returns the torch.cuda.CUDAGraph; replay it with
        `.replay()` on the current stream."""
        torch = self.torch
        s = stream if stream is not None else torch.cuda.Stream(self.device)
        bufs = [self.buffers(ts) for ts in tensor_sets]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for ts, b in zip(tensor_sets, bufs):
                self.launch(ts, s, b)
        return g

    def batched(self, n: int) -> "BatchedExecutable":
        """n independent executions of this call signature in one launch per
        program (many small calls, such as candidate kernels evaluated on
        many inputs).  Each tensor argument becomes one tensor n times its
        size, execution i's copy at element offset i * its size.  Only
        elementwise plans whose every access stays inside its tensor qualify:
        a read past a tensor's end must see the reference's zero fill, not
        the next execution's data."""
        return BatchedExecutable(self, n)

    def check_status(self, value: Optional[int] = None) -> None:
        """Raise for the device status word (read here unless the caller has
        already downloaded it)."""
        if not self.plan.status_check:
            return
        v = int(self.status.item()) if value is None else value
        if v & R.STATUS_NEGATIVE_INDEX:
            self.status.zero_()
            raise IndexError("indirect index from an index view is negative")
        if v & R.STATUS_TIMEOUT:
            self.status.zero_()
            raise RuntimeError("device wait timed out")


class BatchedExecutable:
    """An elementwise plan run as n independent executions per launch (see
    Executable.batched)."""

    def __init__(self, exe: Executable, n: int):
        import copy
        torch = exe.torch
        plan = exe.plan
        if plan.kind != "elementwise" or not plan.launches or n < 1 or \
                any(l.kind != "ew" or l.meta.get("prog") is None or
                    l.meta["prog"].contiguous != 2 for l in plan.launches):
            raise NotImplementedError("batched execution needs an elementwise plan whose "
                                      "accesses stay inside their tensors")
        self.exe, self.n = exe, n
        numel = [b.numel for b in exe.space.buffers]
        self.numel = numel
        self.progs, self.tables = [], []
        for l in plan.launches:
            p = copy.deepcopy(l.meta["prog"])
            t = l.meta["table"]
            units = t.shape[0]
            # column j of the unit table offsets view(s) of one slot; execution
            # i adds i times that slot's tensor size
            add = np.zeros(t.shape[1], np.int64)
            for v in range(p.n_views):
                if p.view[v].unit_col >= 0:
                    add[p.view[v].unit_col] = numel[p.view[v].slot]
            big = (t[None, :, :] + np.arange(n, dtype=np.int64)[:, None, None] * add[None, None, :])
            p.n_units = n * units
            self.progs.append(p)
            self.tables.append(torch.from_numpy(big.reshape(n * units, -1).copy()).to(exe.device))

    def buffers(self, tensors) -> R.KtirBuffers:
        b = R.KtirBuffers()
        for i, t in enumerate(tensors):
            b.base[i] = t.data_ptr()
            b.numel[i] = self.numel[i] * self.n
        return b

    def launch(self, tensors, stream=None, bufs: Optional[R.KtirBuffers] = None) -> None:
        """Enqueue the n executions over `tensors` (one per call tensor, each n
        times its size, in argument address order)."""
        torch = self.exe.torch
        s = stream if stream is not None else torch.cuda.current_stream(self.exe.device)
        sp = C.c_void_p(s.cuda_stream)
        if bufs is None:
            bufs = self.buffers(tensors)
        lib = self.exe.lib
        for p, t in zip(self.progs, self.tables):
            R.check(lib.ktir_ew(C.byref(p), C.byref(bufs), C.c_void_p(t.data_ptr()), sp), "ktir_ew")


class KTIRInterpreter:
    """KTIR interpreter whose execution runs on a B200 (API of ktir_cpu.KTIRInterpreter)."""

    def __init__(self, latency_config: Any = None, trace_latency: bool = False,
                 parser: Optional[KTIRParserBase] = None, device: Any = None,
                 shard: Optional[Tuple[int, int, Any]] = None):
        """`shard=(rank, world, group)` splits every call's core grid across
        `world` GPUs by contiguous core ranges: this process executes only the
        cores of `rank` (programs that need an exchange between shards use the
        torch.distributed `group`).  Tensors this shard does not write come
        back unchanged."""
        self.module: Optional[IRModule] = None
        self.memory: Optional[DeviceMemory] = None
        self.grid_executor = None
        self._parser = parser
        self._latency_config = latency_config
        self._trace_latency = trace_latency
        self._latency_report = None
        self._device = device
        self._shard = shard
        self._cache: Dict[Any, Tuple[Executable, AddressSpace]] = {}
        self.last_executable: Optional[Executable] = None

    # -- loading / inspection -----------------------------------------------------
    def load(self, ktir_source: str) -> None:
        parser = self._parser if self._parser is not None else KTIRParser()
        if "\n" in ktir_source or ktir_source.lstrip().startswith("module"):
            self.module = parser.parse_module(ktir_source)
        else:
            self.module = parser.parse_file(ktir_source)
        self._cache.clear()

    def arg_names(self, func_name: str) -> List[str]:
        if not self.module:
            raise RuntimeError("No module loaded. Call load() first.")
        return self.module.get_function(func_name).arg_names

    def tensor_input_output_sizes(self, func_name: str) -> Dict[str, Dict[str, Any]]:
        if not self.module:
            raise RuntimeError("No module loaded. Call load() first.")
        return self.module.get_function(func_name).tensor_sizes

    def get_latency_report(self):
        if self._latency_config is None:
            return None
        return self._latency_report

    def _prepare_execution(self, grid_shape: Tuple[int, int, int]) -> None:
        self.memory = DeviceMemory(grid_shape[0] * grid_shape[1] * grid_shape[2])
        if self._latency_config is not None:
            from .latency import LatencyReport
            self._latency_report = LatencyReport(self._latency_config, {})

    # -- execution ----------------------------------------------------------------------
    def _device_obj(self):
        torch = R.require_cuda()
        R.load_library()
        if self._device is None:
            self._device = torch.device("cuda", torch.cuda.current_device())
        return torch.device(self._device)

    def _bind(self, func_name: str, kwargs: Dict[str, Any]):
        """Allocate every ndarray argument in the HBM façade (stick-aligned, in
        argument order, as ktir_cpu/interpreter.py:137-160 does)."""
        if not self.module:
            raise RuntimeError("No module loaded. Call load() first.")
        func = self.module.get_function(func_name)
        self._prepare_execution(func.grid)
        declared = func.arg_names
        if kwargs and declared and not any(k in declared for k in kwargs):
            if len(kwargs) == len(declared):
                kwargs = dict(zip(declared, kwargs.values()))
        hbm = self.memory.hbm
        ptrs: Dict[str, Any] = {}
        scalars: Dict[str, Any] = {}
        dts: Dict[str, str] = {}
        for name, v in kwargs.items():
            if isinstance(v, np.ndarray):
                if np.dtype(v.dtype) not in _KTIR_OF:
                    raise ValueError(f"No KTIR dtype for NumPy dtype: {v.dtype!r}")
                stick = hbm.allocate(v.nbytes)
                hbm.attach(stick, v)
                ptrs[name] = stick
                dts[name] = _KTIR_OF[np.dtype(v.dtype)]
            else:
                scalars[name] = v
        return func, kwargs, ptrs, scalars, dts

    def _space(self, ptrs: Dict[str, int]) -> AddressSpace:
        space = AddressSpace()
        names = {v * STICK: k for k, v in ptrs.items()}
        for addr, fac, key in self.memory.allocations():
            arr = fac.allocs[key]
            label = names.get(addr, f"hbm@0x{addr:x}" if fac is self.memory.hbm else
                              f"lx@0x{key:x}")
            space.add_fixed(label, addr, arr.nbytes, arr.dtype, arr.shape)
        return space

    def execute_function(self, func_name: str, **kwargs) -> Dict[str, np.ndarray]:
        func, kwargs, ptrs, scalars, dts = self._bind(func_name, kwargs)
        hbm = self.memory.hbm
        exe, order = self._executable(func_name, ptrs, scalars)
        if self._latency_config is not None:
            # charged on the call's inputs, before the device writes anything
            self._latency_report = exe.latency_tape.report(
                self._latency_config, self._trace_latency, self._index_reader())
        self.run_host(exe, order)
        out = {}
        for name, v in kwargs.items():
            if isinstance(v, np.ndarray):
                out[name] = hbm.allocs[ptrs[name] * STICK].reshape(v.shape)
        return out

    def estimate_latency(self, func_name: str, **kwargs):
        """The latency report of one call, computed on the host without running
        it (no GPU needed); `latency_config` defaults to HardwareConfig()."""
        from .latency import HardwareConfig, LatencyTape
        func, kwargs, ptrs, scalars, dts = self._bind(func_name, kwargs)
        tape = LatencyTape()
        Tracer(func, self._space(ptrs), scalars, ptrs, latency=tape).run()
        cfg = self._latency_config if self._latency_config is not None else HardwareConfig()
        return tape.report(cfg, self._trace_latency, self._index_reader())

    def _index_reader(self):
        """Values of index tensors at byte addresses, from the host copies of the
        call's allocations (zero outside every allocation, like a read past the
        end of one)."""
        from .trace import np_dtype
        allocs = [(addr, fac.allocs[key].view(np.uint8).reshape(-1))
                  for addr, fac, key in self.memory.allocations()]

        def read(addrs: np.ndarray, dtype: str) -> np.ndarray:
            dt = np_dtype(dtype)
            raw = np.zeros((addrs.size, dt.itemsize), np.uint8)
            for base, b in allocs:
                sel = (addrs >= base) & (addrs + dt.itemsize <= base + b.size)
                if sel.any():
                    rel = addrs[sel] - base
                    raw[sel] = b[rel[:, None] + np.arange(dt.itemsize)]
            return raw.reshape(-1).view(dt)
        return read

    def _executable(self, func_name: str, ptrs: Dict[str, int], scalars: Dict[str, Any]):
        allocs = [(a, fac.allocs[k]) for a, fac, k in self.memory.allocations()]
        key = (func_name, tuple((a, arr.nbytes, str(arr.dtype)) for a, arr in allocs),
               tuple(sorted((k, repr(v)) for k, v in scalars.items())),
               tuple(sorted(ptrs.items())))
        hit = self._cache.get(key)
        if hit is not None:
            self.last_executable = hit[0]
            return hit
        if len(allocs) > R.ARENA_SLOT - 1:
            raise NotImplementedError(f"at most {R.ARENA_SLOT - 1} tensors per call")
        device = self._device_obj()
        func = self.module.get_function(func_name)
        space = self._space(ptrs)
        from .latency import LatencyTape
        from .rewrite import attention_rewrites
        slots = {b.index: b.index for b in space.buffers}
        rewrites = attention_rewrites(func)
        tape = LatencyTape() if self._latency_config is not None else None
        trace = Tracer(func, space, scalars, ptrs, rewrites=rewrites,
                       latency=None if rewrites else tape).run()
        plan = Lowerer(trace, device, slots, self._shard).lower()
        if rewrites and plan.kind != "attention":
            # the rewritten loops did not form a whole attention problem the
            # tensor-core kernel covers: trace the loops op by op instead
            trace = Tracer(func, space, scalars, ptrs, latency=tape).run()
            plan = Lowerer(trace, device, slots, self._shard).lower()
        elif rewrites and tape is not None:
            # rewritten loops are not traced op by op: one more pass for the tape
            Tracer(func, space, scalars, ptrs, latency=tape).run()
        exe = Executable(plan, space, device, func.grid)
        exe.latency_tape = tape
        entry = (exe, [a for a, _ in allocs])
        self._cache[key] = entry
        self.last_executable = exe
        return entry

    def run_host(self, exe: Executable, order: List[int]) -> None:
        """Upload the allocations, run the plan, read back what the plan writes.

        Every allocation of the façade is replaced by a new array holding its
        contents after the call (the caller's input arrays are never written).
        Each allocation gets a page-locked buffer from a pool for the call: the
        library copies the caller's array into it in chunks on its worker
        threads, DMAs each chunk to the device as soon as it is staged, and
        after the plan DMAs what the plan wrote back into the same buffer,
        which is then the returned array (an allocation the plan does not
        write comes back as its staged copy).  A buffer returns to the pool
        once no array refers to it any more.  Buffers the plan overwrites
        entirely without reading are not uploaded.  When the pool is at its
        size limit, the call stages through the Executable's own pinned
        buffers and copies the results into new arrays instead.
        """
        torch = exe.torch
        lib = exe.lib
        where = {a: (fac, k) for a, fac, k in self.memory.allocations()}
        arrays = [where[a][0].allocs[where[a][1]] for a in order]
        if exe.dev_tensors is None:
            exe.dev_tensors = [torch.empty(arr.nbytes + 16, dtype=torch.uint8, device=exe.device)
                               for arr in arrays]
            exe.bufs = exe.buffers(exe.dev_tensors)
            exe.status_pinned = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        stream = torch.cuda.current_stream(exe.device)
        sp = C.c_void_p(stream.cuda_stream)
        dev = exe.device.index if exe.device.index is not None else torch.cuda.current_device()
        written = exe.plan.info.get("written")
        skip = exe.plan.info.get("overwritten", set())
        src = [np.ascontiguousarray(arr).view(np.uint8).reshape(-1) for arr in arrays]
        n = len(order)
        staged = _PINNED.take([s_.size for s_ in src], torch)
        if staged is None:
            if exe.pinned is None:
                exe.pinned = [torch.empty(max(s_.size, 1), dtype=torch.uint8, pin_memory=True)
                              for s_ in src]
            pinned = [t.data_ptr() for t in exe.pinned]
            results = [np.empty(s_.size, np.uint8) for s_ in src]
        else:
            pinned = [a.ctypes.data for _, a in staged]
            results = [a[:s_.size] for (_, a), s_ in zip(staged, src)]
        up = [i for i in range(n) if i not in skip and src[i].size]
        # a split plan may read only parts of some tensors (its share of them)
        ranges = exe.plan.info.get("upload_ranges", {}) if self._shard is not None else {}
        xfer = []
        for i in up:
            for off, nb in ranges.get(i, [(0, src[i].size)]):
                xfer.append((src[i].ctypes.data + off, pinned[i] + off,
                             exe.dev_tensors[i].data_ptr() + off, nb))
        xs = (R.KtirHostXfer * max(1, len(xfer)))()
        for k, (h, p_, d_, nb) in enumerate(xfer):
            xs[k].host, xs[k].pinned, xs[k].device, xs[k].bytes = h, p_, d_, nb
        R.check(lib.ktir_host_upload(xs, len(xfer), dev, sp), "ktir_host_upload")
        if exe.plan.status_check:
            exe.status.zero_()
        merge = self._shard is not None and self._shard[1] > 1
        if merge:
            back_all = [i for i in range(n) if (written is None or i in written) and src[i].size]
            before = {i: exe.dev_tensors[i][:src[i].size].clone() for i in back_all}
        exe.launch(exe.dev_tensors, stream, exe.bufs)
        if merge:
            self._merge_shards(exe, before, sp)
        back = [i for i in range(n) if (written is None or i in written) and src[i].size]
        status = np.zeros(1, np.int32)
        ys = (R.KtirHostXfer * (len(back) + 1))()
        for k, i in enumerate(back):
            ys[k].host, ys[k].pinned = results[i].ctypes.data, pinned[i]
            ys[k].device, ys[k].bytes = exe.dev_tensors[i].data_ptr(), src[i].size
        n_y = len(back)
        if exe.plan.status_check:
            ys[n_y].host, ys[n_y].pinned = status.ctypes.data, exe.status_pinned.data_ptr()
            ys[n_y].device, ys[n_y].bytes = exe.status.data_ptr(), 4
            n_y += 1
        # allocations neither written back nor already staged whole into their result
        rest = [i for i in range(n) if i not in back and src[i].size
                and (staged is None or i not in up or i in ranges)]
        cs = (R.KtirHostCopy * max(1, len(rest)))()
        for k, i in enumerate(rest):
            cs[k].dst, cs[k].src, cs[k].bytes = results[i].ctypes.data, src[i].ctypes.data, src[i].size
        R.check(lib.ktir_host_download(ys, n_y, cs, len(rest), dev, sp), "ktir_host_download")
        exe.check_status(int(status[0]))
        for i, addr in enumerate(order):
            fac, k = where[addr]
            fac.allocs[k] = results[i].view(arrays[i].dtype)
            fac.borrowed.add(k)
        exe.last_h2d_bytes = sum(x[3] for x in xfer)
        exe.last_d2h_bytes = sum(src[i].size for i in back)

    def _merge_shards(self, exe: Executable, before, sp) -> None:
        """Make every rank's tensors whole after a split call: each rank wrote
        only its cores' elements, every other element still holds the uploaded
        value (the same on every rank).  The byte differences from the upload,
        summed over the ranks modulo 256 (NCCL all-reduce of uint8; at most one
        rank changes a given byte), added back to the upload give every rank
        the combined result, bit for bit."""
        import torch.distributed as dist
        lib = exe.lib
        group = self._shard[2]
        for i, orig in before.items():
            cur = exe.dev_tensors[i][:orig.numel()]
            delta = exe.torch.empty_like(orig)
            R.check(lib.ktir_bytes_delta(C.c_void_p(delta.data_ptr()), C.c_void_p(cur.data_ptr()),
                                         C.c_void_p(orig.data_ptr()), orig.numel(), 1, sp),
                    "ktir_bytes_delta")
            dist.all_reduce(delta, op=dist.ReduceOp.SUM, group=group)
            R.check(lib.ktir_bytes_delta(C.c_void_p(cur.data_ptr()), C.c_void_p(orig.data_ptr()),
                                         C.c_void_p(delta.data_ptr()), orig.numel(), 0, sp),
                    "ktir_bytes_delta")



class _PinnedPool:
    """Page-locked host buffers handed out as call results and reused once
    nothing refers to them (every view of a buffer holds a reference to it,
    so an idle buffer is one only the pool holds).  Buffers are kept per
    size; the pool stops growing at KTIR_PINNED_POOL_BYTES (default 8 GiB)."""

    def __init__(self) -> None:
        import threading
        self.free: Dict[int, List[List[Any]]] = {}
        self.bytes = 0
        self.limit = int(os.environ.get("KTIR_PINNED_POOL_BYTES", str(8 << 30)))
        self.lock = threading.Lock()

    def take(self, sizes: List[int], torch) -> Optional[List[Tuple[Any, np.ndarray]]]:
        """One idle buffer per size (all or none); safe to call from several threads."""
        with self.lock:
            return self._take(sizes, torch)

    def _take(self, sizes: List[int], torch) -> Optional[List[Tuple[Any, np.ndarray]]]:
        picked: List[List[Any]] = []
        new_bytes = 0
        for nb in sizes:
            nb = max(int(nb), 1)
            entry = None
            for e in self.free.get(nb, []):
                # held by the pool's list and by getrefcount's argument only
                if not e[2] and sys.getrefcount(e[1]) == 2:
                    entry = e
                    break
            if entry is None:
                new_bytes += nb
                entry = [None, None, False, nb]
            entry[2] = True
            picked.append(entry)
        if self.bytes + new_bytes > self.limit:
            for e in picked:
                e[2] = False
            return None
        out = []
        for e in picked:
            if e[0] is None:
                t = torch.empty(e[3], dtype=torch.uint8, pin_memory=True)
                e[0], e[1] = t, t.numpy()
                self.free.setdefault(e[3], []).append(e)
                self.bytes += e[3]
            e[2] = False
            out.append((e[0], e[1]))
        return out


_PINNED = _PinnedPool()


