"""KTIR MLIR text parser.

Reads the textual form of KTDP kernels (``func.func`` bodies made of
``ktdp`` / ``arith`` / ``math`` / ``linalg`` / ``scf`` / ``tensor`` ops) into
:mod:`ktir_cpu_b200.ir`.  Accepts the same surface syntax the reference's
regex parser does (ktir_cpu/parser.py:85-511 and the per-dialect parsers in
ktir_cpu/dialects/*_ops.py), with a different structure: a bracket-aware
statement splitter, explicit region extraction (a ``{...}`` block whose body
holds SSA names or a ``^bb`` label is a region, anything else is an attribute
dictionary — the same rule as ktir_cpu/parser.py:413-435), then one small
parser per op family that fills a normalised attribute dictionary.

Module-scope aliases (``#name = affine_set<...>``) are collected first and
substituted where an attribute value names them (ktir_cpu/parser.py:97-107).
"""

from __future__ import annotations

import re
from typing import Any, Callable, Dict, List, Optional, Tuple

from .affine import (AffineMap, BoxSet, parse_affine_map, parse_affine_set, parse_affine_set_raw,
                     parse_expr)
from .ir import IRFunction, IRModule, Operation, Region

SSA = r"%[A-Za-z0-9_$.#]+"
_SSA_RE = re.compile(SSA)
_RESULTS_RE = re.compile(
    r"^\s*(%[\w$.]+(?::\d+)?(?:\s*,\s*%[\w$.]+)*)\s*=(?!=)\s*")
_STMT_START = re.compile(
    r"^(?:%[\w$.]+(?::\d+)?(?:\s*,\s*%[\w$.]+)*\s*=(?!=)|[a-z_][\w]*\.[\w.]+|return\b|\^)")
_OPEN = "({["
_CLOSE = ")}]"


class KTIRParseError(ValueError):
    pass


def _is_angle_open(text: str, i: int) -> bool:
    return text[i] == "<" and not (i + 1 < len(text) and text[i + 1] == "=")


def _is_angle_close(text: str, i: int) -> bool:
    if text[i] != ">":
        return False
    if i > 0 and text[i - 1] == "-":
        return False
    return not (i + 1 < len(text) and text[i + 1] == "=")


# ---------------------------------------------------------------------------
# Text helpers
# ---------------------------------------------------------------------------

def strip_comments(text: str) -> str:
    return re.sub(r"//[^\n]*", "", text)


def find_close(text: str, i: int) -> int:
    """Index of the bracket closing the one at text[i] ((), [], {} or <>)."""
    pairs = {"(": ")", "[": "]", "{": "}", "<": ">"}
    open_ch = text[i]
    close_ch = pairs[open_ch]
    depth = 0
    j = i
    while j < len(text):
        ch = text[j]
        if ch == open_ch and (open_ch != "<" or _is_angle_open(text, j)):
            depth += 1
        elif ch == close_ch:
            if close_ch == ">" and not _is_angle_close(text, j):
                j += 1
                continue
            depth -= 1
            if depth == 0:
                return j
        j += 1
    raise KTIRParseError(f"unbalanced {open_ch!r} in {text[i:i + 80]!r}")


def split_top(text: str, sep: str = ",") -> List[str]:
    parts: List[str] = []
    depth = 0
    cur = []
    i = 0
    while i < len(text):
        ch = text[i]
        if ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        elif _is_angle_open(text, i):
            depth += 1
        elif _is_angle_close(text, i):
            depth -= 1
        if ch == sep and depth == 0:
            parts.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
        i += 1
    if cur or parts:
        parts.append("".join(cur))
    return [p.strip() for p in parts if p.strip()]


def ssa_names(text: str) -> List[str]:
    return _SSA_RE.findall(text)


def parse_type(t: str) -> Dict[str, Any]:
    """tensor<2x3xf16> / memref<?x4xf32> / !ktdp.access_tile<4xindex> / f16 / index."""
    t = t.strip()
    m = re.match(r"^(tensor|memref|!ktdp\.access_tile|vector)<(.*)>$", t, re.S)
    if m:
        kind = m.group(1)
        inner = m.group(2).split(",")[0].strip()
        dims: List[Any] = []
        rest = inner
        while True:
            mm = re.match(r"^\s*(\d+|\?)\s*x", rest)
            if not mm:
                break
            dims.append(None if mm.group(1) == "?" else int(mm.group(1)))
            rest = rest[mm.end():]
        return {"kind": kind, "shape": tuple(dims), "dtype": rest.strip()}
    return {"kind": "scalar", "shape": (), "dtype": t}


def parse_number(s: str, dtype: Optional[str] = None) -> Any:
    """Integer / float / hex literal.  Hex with a float type is an IEEE bit
    pattern (ktir_cpu/parser_utils.py:86-127)."""
    import numpy as np
    s = s.strip()
    if s in ("true", "false"):
        return s == "true"
    neg = s.startswith("-")
    body = s[1:] if neg else s
    if body.lower().startswith("0x"):
        bits = int(body, 16)
        if dtype == "f32":
            v = float(np.array([bits & 0xFFFFFFFF], np.uint32).view(np.float32)[0])
        elif dtype in ("f16", "fp16", "float16"):
            v = float(np.array([bits & 0xFFFF], np.uint16).view(np.float16)[0])
        elif dtype == "bf16":
            v = float(np.array([(bits & 0xFFFF) << 16], np.uint32).view(np.float32)[0])
        else:
            v = bits
        return -v if neg else v
    try:
        return int(s)
    except ValueError:
        pass
    try:
        return float(s)
    except ValueError:
        raise KTIRParseError(f"bad numeric literal {s!r}")


def attr_dict(text: str, aliases: Dict[str, str]) -> Dict[str, str]:
    """Parse the first top-level ``{ key = value, ... }`` block into raw strings."""
    i = text.find("{")
    if i < 0:
        return {}
    j = find_close(text, i)
    body = text[i + 1:j]
    out: Dict[str, str] = {}
    for item in split_top(body):
        if "=" not in item:
            continue
        k, v = item.split("=", 1)
        v = v.strip()
        if v.startswith("#") and v in aliases:
            v = aliases[v]
        out[k.strip()] = v
    return out


def remove_attr_dicts(text: str) -> str:
    out = []
    i = 0
    while i < len(text):
        if text[i] == "{":
            j = find_close(text, i)
            i = j + 1
            continue
        out.append(text[i])
        i += 1
    return "".join(out)


def after_colon_types(text: str) -> List[str]:
    """Types after the last top-level ':' (comma separated)."""
    t = remove_attr_dicts(text)
    depth = 0
    last = -1
    for i, ch in enumerate(t):
        if ch in "([" or _is_angle_open(t, i):
            depth += 1
        elif ch in ")]" or _is_angle_close(t, i):
            depth -= 1
        elif ch == ":" and depth == 0:
            last = i
    if last < 0:
        return []
    return split_top(t[last + 1:])


def arrow_type(text: str) -> Optional[str]:
    t = remove_attr_dicts(text)
    idx = t.rfind("->")
    if idx < 0:
        return None
    return t[idx + 2:].strip().strip("()").strip()


def bracket_after(text: str, key: str) -> Optional[str]:
    m = re.search(re.escape(key.rstrip(" =:")) + r"\s*[=:]?\s*\[", text)
    if not m:
        return None
    i = m.end() - 1
    j = find_close(text, i)
    return text[i + 1:j]


def paren_after(text: str, key: str) -> Optional[str]:
    m = re.search(r"\b" + re.escape(key) + r"\s*\(", text)
    if not m:
        return None
    i = m.end() - 1
    j = find_close(text, i)
    return text[i + 1:j]


def _ints_or_names(s: str) -> List[Any]:
    out: List[Any] = []
    for tok in split_top(s):
        tok = tok.strip()
        try:
            out.append(int(tok))
        except ValueError:
            out.append(tok)
    return out


# ---------------------------------------------------------------------------
# Statement splitting and region extraction
# ---------------------------------------------------------------------------

def _depth_delta(line: str) -> int:
    d = 0
    for ch in line:
        if ch in _OPEN:
            d += 1
        elif ch in _CLOSE:
            d -= 1
    return d


def split_statements(body: str) -> List[str]:
    stmts: List[str] = []
    cur: List[str] = []
    depth = 0
    for raw in body.split("\n"):
        line = raw.strip()
        if not line:
            continue
        if cur and depth == 0 and _STMT_START.match(line) and not line.startswith("->") \
                and not cur[-1].endswith("="):
            stmts.append(" \n".join(cur))
            cur = []
        cur.append(line)
        depth += _depth_delta(line)
    if cur:
        stmts.append(" \n".join(cur))
    return stmts


def _is_region_body(inner: str) -> bool:
    return "%" in inner or "^" in inner


def extract_regions(text: str) -> Tuple[str, List[Tuple[str, str]]]:
    """Pull ``{...}`` region bodies out of a statement.

    Returns (text_without_regions, [(pre_args_text, body_text), ...]) where
    pre_args_text is a ``(%a: f32, %b: f32)`` block-argument list written just
    before the region (the explicit linalg.reduce form), if any.
    """
    out: List[str] = []
    regions: List[Tuple[str, str]] = []
    i = 0
    while i < len(text):
        ch = text[i]
        if ch == "{":
            j = find_close(text, i)
            inner = text[i + 1:j]
            if _is_region_body(inner):
                pre = ""
                joined = "".join(out).rstrip()
                m = re.search(r"\((\s*%[\w$.]+\s*:[^()]*)\)\s*$", joined)
                if m and not re.search(r"(ins|outs|iter_args|intermediate_variables)\s*$",
                                       joined[:m.start()].rstrip()):
                    pre = m.group(1)
                    out = list(joined[:m.start()])
                regions.append((pre, inner))
                out.append(" ")
            else:
                out.append(text[i:j + 1])
            i = j + 1
            continue
        out.append(ch)
        i += 1
    return "".join(out), regions


# ---------------------------------------------------------------------------
# Parser
# ---------------------------------------------------------------------------

OpParser = Callable[["KTIRParser", str, List[str], str, List[Region]], Operation]
_PARSERS: Dict[str, OpParser] = {}


def _op(*names: str):
    def deco(fn):
        for n in names:
            _PARSERS[n] = fn
        return fn
    return deco


class KTIRParserBase:
    """Parser protocol: anything with parse_module(str) -> IRModule."""

    def parse_module(self, mlir_text: str) -> IRModule:  # pragma: no cover - interface
        raise NotImplementedError

    def parse_file(self, filepath: str) -> IRModule:
        with open(filepath) as f:
            return self.parse_module(f.read())


class KTIRParser(KTIRParserBase):
    def __init__(self) -> None:
        self.aliases: Dict[str, str] = {}

    # -- module / function -------------------------------------------------
    def parse_module(self, mlir_text: str) -> IRModule:
        text = strip_comments(mlir_text)
        module = IRModule()
        self.aliases = {}
        for m in re.finditer(r"^\s*(#[\w.]+)\s*=\s*", text, re.M):
            rest = text[m.end():]
            value = self._alias_value(rest)
            self.aliases[m.group(1)] = value
        module.aliases = dict(self.aliases)
        for m in re.finditer(r"func\.func\s+(?:private\s+)?@([\w$.]+)\s*\(", text):
            name = m.group(1)
            lp = m.end() - 1
            rp = find_close(text, lp)
            args = self._parse_args(text[lp + 1:rp])
            pos = rp + 1
            header_extra = ""
            body = None
            while pos < len(text):
                if text.startswith("attributes", pos):
                    k = text.index("{", pos)
                    j = find_close(text, k)
                    header_extra += text[pos:j + 1]
                    pos = j + 1
                    continue
                ch = text[pos]
                if ch == "{":
                    j = find_close(text, pos)
                    body = text[pos + 1:j]
                    break
                if ch == "}":
                    break
                header_extra += ch
                pos += 1
            if body is None:
                continue
            grid = self._grid(header_extra)
            ops = self.parse_block(body)
            module.add_function(IRFunction(name=name, arguments=args, operations=ops, grid=grid))
        return module

    def _alias_value(self, rest: str) -> str:
        m = re.match(r"(affine_set|affine_map)\s*<", rest)
        if m:
            i = m.end() - 1
            j = find_close(rest, i)
            return rest[:j + 1].strip()
        return rest.split("\n", 1)[0].strip()

    @staticmethod
    def _parse_args(text: str) -> List[Tuple[str, str]]:
        args = []
        for part in split_top(text):
            m = re.match(r"(%[\w$.]+)\s*:\s*(.+)$", part.strip(), re.S)
            if m:
                args.append((m.group(1), m.group(2).strip()))
        return args

    @staticmethod
    def _grid(header: str) -> Tuple[int, int, int]:
        m = re.search(r"grid\s*=\s*\[([^\]]*)\]", header)
        if not m:
            return (1, 1, 1)
        vals = [int(v) for v in m.group(1).replace(" ", "").split(",") if v]
        vals = (vals + [1, 1, 1])[:3]
        return (vals[0], vals[1], vals[2])

    # -- blocks ------------------------------------------------------------
    def parse_block(self, body: str) -> List[Operation]:
        ops: List[Operation] = []
        for stmt in split_statements(body):
            op = self.parse_statement(stmt)
            if op is not None:
                ops.append(op)
        return ops

    def parse_region(self, pre: str, body: str) -> Region:
        args: List[Tuple[str, str]] = []
        label = False
        if pre:
            args = self._parse_args(pre)
        stripped = body.strip()
        m = re.match(r"^\^[\w]+\s*(\(([^)]*)\))?\s*:", stripped)
        if m:
            if m.group(2):
                args = self._parse_args(m.group(2))
                label = True
            stripped = stripped[m.end():]
        return Region(args=args, ops=self.parse_block(stripped), label=label)

    def parse_statement(self, stmt: str) -> Optional[Operation]:
        text, raw_regions = extract_regions(stmt)
        text = " ".join(text.split())
        if not text:
            return None
        if text.startswith("^"):
            return None  # stray block label; handled by parse_region
        results: List[str] = []
        m = _RESULTS_RE.match(text)
        if m:
            lhs = m.group(1)
            mb = re.fullmatch(r"(%[\w$.]+):(\d+)", lhs.strip())
            if mb:
                results = [f"{mb.group(1)}#{i}" for i in range(int(mb.group(2)))]
            else:
                results = [p.strip() for p in lhs.split(",")]
            text = text[m.end():]
        regions = [self.parse_region(pre, body) for pre, body in raw_regions]
        # infix index arithmetic shorthand: %r = %a * %b : index
        mi = re.match(r"^(%[\w$.]+)\s*([*+\-])\s*(%[\w$.]+)\s*:\s*(\S+)", text)
        if mi:
            op_type = {"*": "arith.muli", "+": "arith.addi", "-": "arith.subi"}[mi.group(2)]
            return Operation(op_type, results, [mi.group(1), mi.group(3)], {},
                             [mi.group(4)], [], stmt)
        mo = re.match(r"^([\w.]+)", text)
        if not mo:
            raise KTIRParseError(f"cannot parse statement: {stmt!r}")
        op_type = mo.group(1)
        rest = text[mo.end():].strip()
        if op_type == "func.return":
            op_type = "return"
        fn = _PARSERS.get(op_type)
        if fn is None:
            for prefix in ("arith.", "math."):
                if op_type.startswith(prefix):
                    fn = _PARSERS["__elementwise__"]
        if fn is None:
            fn = _PARSERS["__generic__"]
        op = fn(self, op_type, results, rest, regions)
        op.text = stmt
        return op

    def alias(self, v: str) -> str:
        v = v.strip()
        return self.aliases.get(v, v)


# ---------------------------------------------------------------------------
# Per-op parsers
# ---------------------------------------------------------------------------

def _mk(op_type, results, operands, attrs, types=None, regions=None) -> Operation:
    return Operation(op_type, list(results), list(operands), attrs, list(types or []),
                     list(regions or []))


@_op("__generic__")
def _p_generic(p, op_type, results, rest, regions):
    operands = ssa_names(remove_attr_dicts(rest).split(":")[0])
    types = after_colon_types(rest)
    attrs: Dict[str, Any] = {}
    arr = arrow_type(rest)
    if arr:
        types = [arr]
    return _mk(op_type, results, operands, attrs, types, regions)


_CMP_PRED = re.compile(r"^(\w+)\s*,")


@_op("__elementwise__")
def _p_elementwise(p, op_type, results, rest, regions):
    attrs: Dict[str, Any] = {}
    body = rest
    if op_type in ("arith.cmpi", "arith.cmpf"):
        m = _CMP_PRED.match(rest)
        if not m:
            raise KTIRParseError(f"{op_type}: missing predicate in {rest!r}")
        attrs["predicate"] = m.group(1)
        body = rest[m.end():]
    # casts: "%a : T1 to T2"
    mt = re.search(r":\s*(.+?)\s+to\s+(.+)$", remove_attr_dicts(body))
    if mt:
        attrs["src_type"] = mt.group(1).strip()
        attrs["dst_type"] = mt.group(2).strip()
        types = [mt.group(2).strip()]
    else:
        types = after_colon_types(body)
    no_attr = remove_attr_dicts(body)
    operand_text = no_attr.split(":")[0]
    # drop fastmath<...> style attributes
    operand_text = re.sub(r"\bfastmath\s*<[^>]*>", "", operand_text)
    operands = ssa_names(operand_text)
    return _mk(op_type, results, operands, attrs, types[-1:] if types else [], regions)


@_op("arith.constant")
def _p_constant(p, op_type, results, rest, regions):
    attrs: Dict[str, Any] = {}
    r = rest.strip()
    mb = re.match(r"^\{(.*)\}\s*:\s*(.+)$", r, re.S)
    if mb:
        r = mb.group(1).strip()
        m2 = re.match(r"^(?:value\s*=\s*)?(.*?)\s*:\s*[^:]+$", r)
        if m2:
            r = m2.group(1) + " : " + mb.group(2)
    md = re.match(r"^dense<(.*)>\s*:\s*(.+)$", r, re.S)
    if md:
        ty = parse_type(md.group(2))
        payload = md.group(1).strip()
        dtype = ty["dtype"]
        if payload.startswith("["):
            flat = payload.replace("[", " ").replace("]", " ")
            vals = [parse_number(v, dtype) for v in flat.split(",") if v.strip()]
            attrs.update(value=vals, dense_list=True)
        else:
            attrs["value"] = parse_number(payload, dtype)
        attrs.update(shape=tuple(ty["shape"]), dtype=dtype, is_tensor=True)
        return _mk(op_type, results, [], attrs, [md.group(2).strip()])
    ms = re.match(r"^(\S+)\s*:\s*(.+)$", r)
    if not ms:
        raise KTIRParseError(f"arith.constant: cannot parse {rest!r}")
    ty = parse_type(ms.group(2))
    if ty["kind"] == "tensor":
        attrs.update(value=parse_number(ms.group(1), ty["dtype"]), shape=tuple(ty["shape"]),
                     dtype=ty["dtype"], is_tensor=True)
    else:
        attrs.update(value=parse_number(ms.group(1), ty["dtype"]), dtype=ty["dtype"])
    return _mk(op_type, results, [], attrs, [ms.group(2).strip()])


@_op("ktdp.get_compute_tile_id")
def _p_tile_id(p, op_type, results, rest, regions):
    types = after_colon_types(rest)
    if types and len(types) != len(results):
        raise KTIRParseError(
            f"ktdp.get_compute_tile_id: {len(results)} result(s) but {len(types)} type(s)")
    return _mk(op_type, results, [], {}, types)


@_op("ktdp.coreid")
def _p_coreid(p, op_type, results, rest, regions):
    return _mk(op_type, results, ssa_names(rest.split(":")[0]), {}, after_colon_types(rest))


@_op("ktdp.construct_memory_view")
def _p_memview(p, op_type, results, rest, regions):
    ptr = ssa_names(rest)[0]
    sizes_txt = bracket_after(rest, "sizes:")
    strides_txt = bracket_after(rest, "strides:")
    mref = re.search(r"memref<([^>]*)>", remove_attr_dicts(rest))
    if not mref:
        raise KTIRParseError("construct_memory_view: could not parse dtype from memref<> type")
    mty = parse_type("memref<" + mref.group(1) + ">")
    dims = list(mty["shape"])
    if not dims:
        raise KTIRParseError(f"construct_memory_view: memref<{mref.group(1)}> has no dimensions")
    if sizes_txt is not None:
        sizes = _ints_or_names(sizes_txt)
        if len(sizes) != len(dims):
            raise KTIRParseError("construct_memory_view: sizes count does not match memref rank")
        for s, d in zip(sizes, dims):
            if d is not None and isinstance(s, int) and s != d:
                raise KTIRParseError(f"construct_memory_view: size {s} does not match memref dim {d}")
            if d is None and isinstance(s, int):
                raise KTIRParseError("construct_memory_view: dynamic dim needs an SSA size")
        shape = tuple(sizes)
    else:
        if any(d is None for d in dims):
            raise KTIRParseError("construct_memory_view: dynamic dims need sizes:")
        shape = tuple(dims)
    strides = _ints_or_names(strides_txt) if strides_txt is not None else [1]
    attrs: Dict[str, Any] = {"shape": shape, "strides": strides, "dtype": mty["dtype"],
                             "memory_space": "HBM"}
    mm = re.search(r"#ktdp\.spyre_memory_space<\s*(\w+)(?:\s*,\s*core\s*=\s*(\d+))?\s*>", rest)
    if mm:
        attrs["memory_space"] = mm.group(1)
        if mm.group(2) is not None:
            attrs["lx_core_id"] = int(mm.group(2))
    ad = attr_dict(rest, p.aliases)
    if "coordinate_set" in ad and ad["coordinate_set"].startswith("affine_set"):
        attrs["coordinate_set"] = parse_affine_set(ad["coordinate_set"])
    operands = [ptr] + [s for s in shape if isinstance(s, str)] + \
        [s for s in strides if isinstance(s, str)]
    return _mk(op_type, results, operands, attrs, ["memref<" + mref.group(1) + ">"])


def _access_shape(rest: str) -> Tuple[int, ...]:
    m = re.search(r"!ktdp\.access_tile<([^>]+)>", rest)
    if not m:
        raise KTIRParseError("missing !ktdp.access_tile<> result type")
    mm = re.match(r"^(\d+(?:x\d+)*)x([A-Za-z_]\w*)$", m.group(1).strip())
    if not mm:
        raise KTIRParseError(f"malformed access_tile type {m.group(1)!r}")
    if mm.group(2) != "index":
        raise KTIRParseError(f"access_tile element type must be 'index', got {mm.group(2)!r}")
    return tuple(int(d) for d in mm.group(1).split("x"))


@_op("ktdp.construct_access_tile")
def _p_access_tile(p, op_type, results, rest, regions):
    head = remove_attr_dicts(rest).split(":")[0]
    operands = ssa_names(head)
    shape = _access_shape(rest)
    ad = attr_dict(rest, p.aliases)
    if "base_map" in ad:
        base_map = parse_affine_map(ad["base_map"])
    else:
        n = max(1, len(operands) - 1)
        dl = ", ".join(f"d{i}" for i in range(n))
        base_map = parse_affine_map(f"affine_map<({dl}) -> ({dl})>")
    if "access_tile_set" not in ad:
        raise KTIRParseError("construct_access_tile: access_tile_set is required")
    cset = parse_affine_set(ad["access_tile_set"])
    attrs: Dict[str, Any] = {"shape": shape, "base_map": base_map, "coordinate_set": cset}
    if "access_tile_order" in ad:
        order = parse_affine_map(ad["access_tile_order"])
        if not order.is_identity():
            attrs["coordinate_order"] = order
    return _mk(op_type, results, operands, attrs, [f"!ktdp.access_tile<{shape}>"])


def _subscript(token: str, var_names: List[str]):
    """Parse one indirect-access subscript into an affine expr whose dims are
    the intermediate variables and whose ("ref", %x) leaves are outer SSA
    values (ktir_cpu/dialects/ktdp_helpers.py:113-145 covers the same forms)."""
    t = token.strip()
    dims = {("%" + v): i for i, v in enumerate(var_names)}
    node = parse_expr(t)

    def fix(n):
        if n[0] == "ref" and n[1] in dims:
            return ("d", dims[n[1]])
        return n
    from .affine import substitute_refs
    return substitute_refs(node, fix)


@_op("ktdp.construct_indirect_access_tile")
def _p_indirect(p, op_type, results, rest, regions):
    iv = paren_after(rest, "intermediate_variables")
    if iv is None:
        raise KTIRParseError("construct_indirect_access_tile: missing intermediate_variables")
    var_names = [v.strip().lstrip("%") for v in iv.split(",") if v.strip()]
    m = re.search(r"intermediate_variables\s*\(", rest)
    after = rest[find_close(rest, m.end() - 1) + 1:]
    mp = re.match(r"\s*(%[\w$.]+)\s*\[", after)
    if not mp:
        raise KTIRParseError("construct_indirect_access_tile: missing primary view subscript")
    primary = mp.group(1)
    lb = mp.end() - 1
    sub_txt = after[lb + 1:find_close(after, lb)]
    dims: List[Dict[str, Any]] = []
    operands = [primary]
    for part in split_top(sub_txt):
        part = part.strip()
        if part.startswith("ind("):
            inner = part[4:part.rfind(")")]
            mv = re.match(r"\s*(%[\w$.]+)\s*\[", inner)
            if not mv:
                raise KTIRParseError(f"bad ind() subscript {part!r}")
            ib = mv.end() - 1
            idx_txt = inner[ib + 1:find_close(inner, ib)]
            exprs = [_subscript(e, var_names) for e in split_top(idx_txt)]
            operands.append(mv.group(1))
            dims.append({"kind": "indirect", "view": len(operands) - 2, "exprs": exprs})
        else:
            inner = part
            if inner.startswith("(") and inner.endswith(")"):
                inner = inner[1:-1]
            dims.append({"kind": "direct", "expr": _subscript(inner, var_names)})
    ad = attr_dict(after, p.aliases)
    if "variables_space_set" not in ad:
        raise KTIRParseError("construct_indirect_access_tile: variables_space_set is required")
    attrs: Dict[str, Any] = {
        "shape": _access_shape(rest),
        "var_names": var_names,
        "dims": dims,
        "variables_space_set": parse_affine_set(ad["variables_space_set"]),
    }
    if "variables_space_order" in ad:
        order = parse_affine_map(ad["variables_space_order"])
        if not order.is_identity():
            attrs["variables_space_order"] = order
    return _mk(op_type, results, operands, attrs, [])


@_op("ktdp.load")
def _p_load(p, op_type, results, rest, regions):
    operands = ssa_names(rest.split(":")[0])
    rt = arrow_type(rest)
    attrs: Dict[str, Any] = {}
    if rt:
        ty = parse_type(rt)
        attrs.update(result_shape=tuple(ty["shape"]), result_dtype=ty["dtype"])
    return _mk(op_type, results, operands[:1], attrs, [rt] if rt else [])


@_op("ktdp.store")
def _p_store(p, op_type, results, rest, regions):
    operands = ssa_names(rest.split(":")[0])
    return _mk(op_type, results, operands[:2], {}, [])


def _ins_outs(rest: str) -> Tuple[List[str], List[str], List[str], List[str]]:
    ins = paren_after(rest, "ins") or ""
    outs = paren_after(rest, "outs") or ""

    def split_io(s):
        if ":" in s:
            names, types = s.split(":", 1)
            return ssa_names(names), split_top(types)
        return ssa_names(s), []
    a, at = split_io(ins)
    b, bt = split_io(outs)
    return a, b, at, bt


@_op("linalg.reduce")
def _p_reduce(p, op_type, results, rest, regions):
    ins, outs, _, out_types = _ins_outs(rest)
    attrs: Dict[str, Any] = {"combiner": None}
    mc = re.match(r"^\{\s*([\w.]+)\s*\}", rest.strip())
    if mc:
        attrs["combiner"] = mc.group(1)
    md = bracket_after(rest, "dimensions =") or bracket_after(rest, "dimensions=")
    if md is not None and md.strip():
        attrs["dims"] = [int(x) for x in md.split(",")]
    attrs["outs"] = outs[0] if outs else None
    return _mk(op_type, results, ins[:1], attrs, out_types, regions)


@_op("linalg.generic")
def _p_generic_linalg(p, op_type, results, rest, regions):
    ad = attr_dict(rest, p.aliases)
    maps: List[AffineMap] = []
    if "indexing_maps" in ad:
        raw = ad["indexing_maps"].strip()[1:-1]
        for item in split_top(raw):
            maps.append(parse_affine_map(p.alias(item)))
    ins, outs, in_types, out_types = _ins_outs(rest)
    attrs = {"indexing_maps": maps, "n_ins": len(ins)}
    if "iterator_types" in ad:
        attrs["iterator_types"] = [s.strip().strip('"') for s in
                                   split_top(ad["iterator_types"].strip()[1:-1])]
    return _mk(op_type, results, ins + outs, attrs, out_types, regions)


@_op("linalg.broadcast")
def _p_broadcast(p, op_type, results, rest, regions):
    ins, outs, _, out_types = _ins_outs(rest)
    md = bracket_after(rest, "dimensions")
    dims = [int(x) for x in md.split(",")] if md and md.strip() else []
    return _mk(op_type, results, ins + outs, {"dimensions": dims}, out_types)


@_op("linalg.transpose")
def _p_transpose(p, op_type, results, rest, regions):
    ins, outs, _, out_types = _ins_outs(rest)
    perm = bracket_after(rest, "permutation")
    if perm is None:
        raise KTIRParseError("linalg.transpose: missing permutation")
    return _mk(op_type, results, ins + outs, {"permutation": [int(x) for x in perm.split(",")]},
               out_types)


@_op("linalg.fill", "linalg.matmul", "linalg.batch_matmul", "linalg.add", "linalg.sub",
     "linalg.mul", "linalg.div", "linalg.max", "linalg.exp")
def _p_linalg_named(p, op_type, results, rest, regions):
    ins, outs, _, out_types = _ins_outs(rest)
    return _mk(op_type, results, ins + outs, {"n_ins": len(ins)}, out_types)


@_op("linalg.index")
def _p_index(p, op_type, results, rest, regions):
    m = re.match(r"^(\d+)", rest.strip())
    if not m:
        raise KTIRParseError("linalg.index: missing dimension")
    return _mk(op_type, results, [], {"dim": int(m.group(1))}, ["index"])


@_op("linalg.yield", "scf.yield", "tensor.yield", "return")
def _p_yield(p, op_type, results, rest, regions):
    return _mk(op_type, results, ssa_names(rest.split(":")[0]), {}, [])


def _named_set(p, rest: str, key: str):
    """The affine set written as `key = #alias` or `key = affine_set<...>`."""
    m = re.search(rf"\b{key}\s*=\s*", rest)
    if not m:
        return None
    tail = rest[m.end():].lstrip()
    if tail.startswith("#"):
        name = re.match(r"#[\w$.]+", tail).group(0)
        text = p.alias(name)
    else:
        i = tail.index("<")
        text = tail[:find_close(tail, i) + 1]
    return parse_affine_set_raw(text)


@_op("ktdp.construct_distributed_memory_view")
def _p_dist_view(p, op_type, results, rest, regions):
    """`(%a, %b : memref<..>, memref<..>) : memref<global>` (ktir_cpu/dialects/
    ktdp_ops.py:418-470): partitions, global shape and dtype."""
    body = rest.lstrip()
    if not body.startswith("("):
        raise KTIRParseError("construct_distributed_memory_view: missing operand parenthesis")
    j = find_close(body, 0)
    inner, tail = body[1:j], body[j + 1:]
    operands = ssa_names(inner.split(":")[0])
    m = re.search(r"memref<([^>]+)>", tail)
    if not m:
        raise KTIRParseError("construct_distributed_memory_view: missing result memref type")
    t = parse_type("memref<" + m.group(1) + ">")
    if any(d is None for d in t["shape"]):
        raise KTIRParseError("construct_distributed_memory_view: dynamic global shape")
    return _mk(op_type, results, operands, {"shape": tuple(t["shape"]), "dtype": t["dtype"]},
               ["memref<" + m.group(1) + ">"])


@_op("ktdp.inter_tile_produce")
def _p_inter_produce(p, op_type, results, rest, regions):
    """ktdp.inter_tile_produce (ktir_cpu/dialects/ktdp_ops.py:998-1038)."""
    prod = _named_set(p, rest, "producer_tiles_per_group")
    groups = _named_set(p, rest, "groups")
    if prod is None or groups is None:
        raise KTIRParseError("ktdp.inter_tile_produce: needs producer_tiles_per_group and groups")
    return _mk(op_type, results, [], {"producer_tiles_per_group": prod, "groups": groups}, [],
               regions)


@_op("ktdp.inter_tile_reduce")
def _p_inter_reduce(p, op_type, results, rest, regions):
    """ktdp.inter_tile_reduce (ktir_cpu/dialects/ktdp_ops.py:1171-1227): the future
    operand, the identity operands and the result shape (within-group axes
    collapsed)."""
    m = re.match(r"^\(\s*(%[\w$.]+)\s*\)", rest)
    if not m:
        raise KTIRParseError(f"ktdp.inter_tile_reduce: cannot parse {rest!r}")
    cons = _named_set(p, rest, "consumer_tiles_per_group")
    groups = _named_set(p, rest, "groups")
    if cons is None or groups is None:
        raise KTIRParseError("ktdp.inter_tile_reduce: needs consumer_tiles_per_group and groups")
    attrs: Dict[str, Any] = {"consumer_tiles_per_group": cons, "groups": groups}
    dep = _named_set(p, rest, "producer_dependency_per_consumer")
    if dep is not None:
        attrs["producer_dependency_per_consumer"] = dep
    ident = paren_after(rest, "identity")
    operands = [m.group(1)] + (ssa_names(ident.split(":")[0]) if ident else [])
    arr = arrow_type(rest)
    if arr:
        t = parse_type(arr)
        if t.get("shape") is not None:
            attrs["result_shape"] = tuple(t["shape"])
    return _mk(op_type, results, operands, attrs, [arr] if arr else [], regions)


@_op("ktdp.yield_partial", "ktdp.yield_reduced")
def _p_inter_yield(p, op_type, results, rest, regions):
    return _mk(op_type, results, ssa_names(rest.split(":")[0]), {}, [])


@_op("scf.for")
def _p_for(p, op_type, results, rest, regions):
    m = re.match(r"^(%[\w$.]+)\s*=\s*(%[\w$.]+|-?\d+)\s+to\s+(%[\w$.]+|-?\d+)\s+step\s+"
                 r"(%[\w$.]+|-?\d+)", rest)
    if not m:
        raise KTIRParseError(f"scf.for: cannot parse header {rest!r}")
    ia = paren_after(rest, "iter_args")
    names: List[str] = []
    inits: List[str] = []
    if ia:
        for pair in split_top(ia):
            a, b = pair.split("=", 1)
            names.append(a.strip())
            inits.append(b.strip())
    attrs = {"iter_var": m.group(1), "iter_args": names}
    if not regions:
        raise KTIRParseError("scf.for: missing body region")
    return _mk(op_type, results, [m.group(2), m.group(3), m.group(4)] + inits, attrs, [], regions)


@_op("scf.if")
def _p_if(p, op_type, results, rest, regions):
    ops = ssa_names(rest.split("->")[0])
    return _mk(op_type, results, ops[:1], {}, [], regions)


@_op("tensor.empty")
def _p_empty(p, op_type, results, rest, regions):
    ty = parse_type(after_colon_types(rest)[-1])
    return _mk(op_type, results, [], {"shape": tuple(ty["shape"]), "dtype": ty["dtype"]},
               [after_colon_types(rest)[-1]])


@_op("tensor.splat")
def _p_splat(p, op_type, results, rest, regions):
    ops = ssa_names(rest.split(":")[0])
    types = after_colon_types(rest)
    rt = arrow_type(rest) or (types[-1] if types else None)
    attrs: Dict[str, Any] = {}
    if rt:
        ty = parse_type(rt)
        if ty["kind"] == "tensor":
            attrs.update(shape=tuple(ty["shape"]), dtype=ty["dtype"])
    return _mk(op_type, results, ops[:1], attrs, [rt] if rt else [])


@_op("tensor.extract")
def _p_extract(p, op_type, results, rest, regions):
    m = re.match(r"^(%[\w$.]+)\s*\[([^\]]*)\]", rest.strip())
    if not m:
        return _mk(op_type, results, ssa_names(rest.split(":")[0])[:1], {}, [])
    return _mk(op_type, results, [m.group(1)] + ssa_names(m.group(2)), {}, [])


@_op("tensor.expand_shape", "tensor.collapse_shape", "tensor.reshape")
def _p_reshape(p, op_type, results, rest, regions):
    ops = ssa_names(remove_attr_dicts(rest).split(":")[0])
    types = re.findall(r"tensor<[^>]*>", rest)
    target = tuple(parse_type(types[-1])["shape"]) if types else None
    return _mk(op_type, results, ops[:1], {"target_shape": target}, types[-1:])


@_op("tensor.from_elements")
def _p_from_elements(p, op_type, results, rest, regions):
    ops = ssa_names(rest.split(":")[0])
    ty = parse_type(after_colon_types(rest)[-1])
    return _mk(op_type, results, ops, {"shape": tuple(ty["shape"]), "dtype": ty["dtype"]})


@_op("tensor.generate")
def _p_generate(p, op_type, results, rest, regions):
    types = after_colon_types(rest)
    ty = parse_type(types[-1])
    return _mk(op_type, results, ssa_names(rest.split("{")[0].split(":")[0]),
               {"shape": tuple(ty["shape"]), "dtype": ty["dtype"]}, types[-1:], regions)
