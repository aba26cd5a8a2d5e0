"""KTIR in-memory IR: module, function, operation, region.

Mirrors the reference's container API (ktir_cpu/ir_types.py:374-448:
``IRModule.get_function``, ``IRFunction.arg_names`` / ``grid`` /
``tensor_sizes``) so callers that inspect a loaded module keep working,
with a structure of our own: every operation carries an explicit result
list, parsed attributes and nested regions with their block arguments.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, Iterator, List, Tuple


@dataclass
class Region:
    args: List[Tuple[str, str]] = field(default_factory=list)  # block arguments
    ops: List["Operation"] = field(default_factory=list)
    label: bool = False   # the arguments come from a ``^bb0(...)`` label


def linalg_block_args(region: Region) -> List[str]:
    """Block-argument names of a ``linalg.reduce`` / ``linalg.generic``
    region, found the way the reference finds them
    (ktir_cpu/dialects/linalg_ops.py:30-58): the arguments of a ``^bb0(...)``
    label, else the operands of the region's first op.  An inline
    ``(%in: f32, %out: f32) {`` list is therefore read from the first op: a
    region whose first op is ``arith.mulf %in, %in`` binds ``%in`` twice and
    leaves ``%out`` unbound, as in the reference."""
    if region.label and region.args:
        return [n for n, _ in region.args]
    if region.ops:
        return list(region.ops[0].operands)
    return [n for n, _ in region.args]


@dataclass
class Operation:
    op_type: str
    results: List[str]
    operands: List[str]
    attributes: Dict[str, Any]
    result_types: List[str] = field(default_factory=list)
    regions: List[Region] = field(default_factory=list)
    text: str = ""

    @property
    def result(self):
        """Single result name, a list for multi-result ops, or None."""
        if not self.results:
            return None
        return self.results[0] if len(self.results) == 1 else list(self.results)

    def __repr__(self) -> str:
        lhs = ", ".join(self.results)
        return f"{lhs + ' = ' if lhs else ''}{self.op_type}({', '.join(self.operands)})"


def iter_ops(ops: List[Operation]) -> Iterator[Operation]:
    for op in ops:
        yield op
        for region in op.regions:
            yield from iter_ops(region.ops)


@dataclass
class IRFunction:
    name: str
    arguments: List[Tuple[str, str]]
    operations: List[Operation]
    grid: Tuple[int, int, int] = (1, 1, 1)
    tensor_sizes: Dict[str, Dict[str, Any]] = field(default_factory=dict, init=False)

    def __post_init__(self) -> None:
        # First construct_memory_view per pointer argument fixes the tensor's
        # shape and dtype (reference: ktir_cpu/ir_types.py:413-421).
        for op in iter_ops(self.operations):
            if op.op_type == "ktdp.construct_memory_view" and op.operands:
                arg = op.operands[0].lstrip("%")
                if arg not in self.tensor_sizes:
                    self.tensor_sizes[arg] = {
                        "shape": tuple(op.attributes.get("shape", ())),
                        "dtype": op.attributes.get("dtype", "f16"),
                    }

    @property
    def arg_names(self) -> List[str]:
        return [n.lstrip("%") for n, _ in self.arguments]

    @property
    def num_cores(self) -> int:
        x, y, z = self.grid
        return x * y * z


@dataclass
class IRModule:
    functions: Dict[str, IRFunction] = field(default_factory=dict)
    aliases: Dict[str, str] = field(default_factory=dict)

    def get_function(self, name: str) -> IRFunction:
        if name not in self.functions:
            raise ValueError(f"Function '{name}' not found in module")
        return self.functions[name]

    def add_function(self, func: IRFunction) -> None:
        self.functions[func.name] = func
