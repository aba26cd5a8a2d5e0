"""Affine maps and integer sets for KTIR attributes.

Covers the ``affine_map<...>`` / ``affine_set<...>`` attribute grammar that
KTIR access tiles, memory views and indirect access tiles carry
(reference: ktir_cpu/affine.py:86-508 for the map/set/box semantics,
ktir_cpu/parser_ast.py:179-320 for the expression grammar).

Expressions are plain tuples so they hash and compare structurally:

    ("c", k)            integer constant
    ("d", i)            dimension variable i
    ("s", i)            symbol variable i
    ("ref", "%name")    SSA reference (only inside ktdp subscripts)
    ("+", a, b)  ("-", a, b)  ("neg", a)
    ("*", k, a)         constant coefficient times expression
    ("mod", a, k) ("floordiv", a, k) ("ceildiv", a, k)

Every evaluator accepts either Python ints or NumPy integer arrays for the
dimension values, so a whole variable space (e.g. the 131,072 points of an
indirect gather chunk) is evaluated in one vectorised pass instead of a
Python loop per point.
"""

from __future__ import annotations

import itertools
import re
from dataclasses import dataclass, field
from typing import Any, List, Optional, Sequence, Tuple

import numpy as np

Expr = tuple

# ---------------------------------------------------------------------------
# Tokeniser + recursive-descent parser
# ---------------------------------------------------------------------------

_TOK = re.compile(
    r"\s*(?:(%[A-Za-z_$.][\w$.]*)|([A-Za-z_][\w]*)|(\d+)|(==|>=|<=|->|[-+*(),:\[\]]))"
)


def tokenize(text: str) -> List[str]:
    out: List[str] = []
    pos = 0
    n = len(text)
    while pos < n:
        m = _TOK.match(text, pos)
        if not m or m.end() == pos:
            if text[pos].isspace():
                pos += 1
                continue
            raise ValueError(f"unexpected character {text[pos]!r} in affine text {text!r}")
        tok = m.group(1) or m.group(2) or m.group(3) or m.group(4)
        if tok is None:
            pos = m.end()
            continue
        out.append(tok)
        pos = m.end()
    return out


class _ExprParser:
    """expr := term (('+'|'-') term)* ; term := factor (('*' int)|('mod'|'floordiv'|'ceildiv') int)*"""

    def __init__(self, tokens: List[str], dims: Optional[dict] = None,
                 syms: Optional[dict] = None):
        self.toks = tokens
        self.i = 0
        self.dims = dims or {}
        self.syms = syms or {}

    def peek(self) -> Optional[str]:
        return self.toks[self.i] if self.i < len(self.toks) else None

    def take(self, expect: Optional[str] = None) -> str:
        tok = self.peek()
        if tok is None:
            raise ValueError("unexpected end of affine expression")
        if expect is not None and tok != expect:
            raise ValueError(f"expected {expect!r}, got {tok!r}")
        self.i += 1
        return tok

    def ident_list(self, open_: str, close: str) -> List[str]:
        names: List[str] = []
        self.take(open_)
        while self.peek() != close:
            names.append(self.take())
            if self.peek() == ",":
                self.take(",")
        self.take(close)
        return names

    def expr(self) -> Expr:
        node = self.term()
        while self.peek() in ("+", "-"):
            op = self.take()
            rhs = self.term()
            node = ("+", node, rhs) if op == "+" else ("-", node, rhs)
        return node

    def term(self) -> Expr:
        node = self.unary()
        while True:
            tok = self.peek()
            if tok == "*":
                self.take()
                rhs = self.unary()
                k_l, k_r = _as_const(node), _as_const(rhs)
                if k_l is not None:
                    node = ("*", k_l, rhs)
                elif k_r is not None:
                    node = ("*", k_r, node)
                else:
                    raise ValueError("affine product needs a constant factor")
            elif tok in ("mod", "floordiv", "ceildiv"):
                self.take()
                rhs = self.unary()
                k = _as_const(rhs)
                if k is None or k <= 0:
                    raise ValueError(f"{tok} needs a positive constant divisor")
                node = (tok, node, k)
            else:
                return node

    def unary(self) -> Expr:
        if self.peek() == "-":
            self.take()
            inner = self.unary()
            k = _as_const(inner)
            return ("c", -k) if k is not None else ("neg", inner)
        return self.atom()

    def atom(self) -> Expr:
        tok = self.take()
        if tok == "(":
            node = self.expr()
            self.take(")")
            return node
        if tok.isdigit():
            return ("c", int(tok))
        if tok.startswith("%"):
            return ("ref", tok)
        if tok in self.dims:
            return ("d", self.dims[tok])
        if tok in self.syms:
            return ("s", self.syms[tok])
        if not self.dims and re.fullmatch(r"d\d+", tok):
            return ("d", int(tok[1:]))
        if not self.syms and re.fullmatch(r"s\d+", tok):
            return ("s", int(tok[1:]))
        raise ValueError(f"unknown identifier {tok!r} in affine expression")


def _as_const(node: Expr) -> Optional[int]:
    return node[1] if node[0] == "c" else None


def parse_expr(text: str, dims: Optional[dict] = None, syms: Optional[dict] = None) -> Expr:
    p = _ExprParser(tokenize(text), dims, syms)
    node = p.expr()
    if p.peek() is not None:
        raise ValueError(f"trailing tokens in affine expression {text!r}")
    return node


# ---------------------------------------------------------------------------
# Evaluation (scalar or vectorised)
# ---------------------------------------------------------------------------

def eval_expr(node: Expr, dims: Sequence[Any], syms: Sequence[Any] = (),
              refs: Optional[dict] = None) -> Any:
    tag = node[0]
    if tag == "c":
        return node[1]
    if tag == "d":
        return dims[node[1]]
    if tag == "s":
        return syms[node[1]]
    if tag == "ref":
        if refs is None or node[1] not in refs:
            raise KeyError(f"unresolved SSA reference {node[1]} in affine expression")
        return refs[node[1]]
    if tag == "+":
        return eval_expr(node[1], dims, syms, refs) + eval_expr(node[2], dims, syms, refs)
    if tag == "-":
        return eval_expr(node[1], dims, syms, refs) - eval_expr(node[2], dims, syms, refs)
    if tag == "neg":
        return -eval_expr(node[1], dims, syms, refs)
    if tag == "*":
        return node[1] * eval_expr(node[2], dims, syms, refs)
    if tag == "mod":
        return eval_expr(node[1], dims, syms, refs) % node[2]
    if tag == "floordiv":
        return eval_expr(node[1], dims, syms, refs) // node[2]
    if tag == "ceildiv":
        return -((-eval_expr(node[1], dims, syms, refs)) // node[2])
    raise ValueError(f"bad affine node {node!r}")


def linearize(node: Expr, n_dims: int, n_syms: int = 0):
    """Return (dim_coeffs, sym_coeffs, const) or None if not linear."""
    dc = [0] * n_dims
    sc = [0] * n_syms
    const = [0]

    def walk(n: Expr, k: int) -> bool:
        tag = n[0]
        if tag == "c":
            const[0] += k * n[1]
        elif tag == "d":
            if n[1] >= n_dims:
                return False
            dc[n[1]] += k
        elif tag == "s":
            if n[1] >= n_syms:
                return False
            sc[n[1]] += k
        elif tag == "+":
            return walk(n[1], k) and walk(n[2], k)
        elif tag == "-":
            return walk(n[1], k) and walk(n[2], -k)
        elif tag == "neg":
            return walk(n[1], -k)
        elif tag == "*":
            return walk(n[2], k * n[1])
        else:
            return False
        return True

    return (dc, sc, const[0]) if walk(node, 1) else None


def substitute_refs(node: Expr, fn) -> Expr:
    """Rebuild *node* replacing every ("ref", name) leaf by fn(leaf)."""
    tag = node[0]
    if tag == "ref":
        return fn(node)
    if tag in ("+", "-"):
        return (tag, substitute_refs(node[1], fn), substitute_refs(node[2], fn))
    if tag == "neg":
        return ("neg", substitute_refs(node[1], fn))
    if tag == "*":
        return ("*", node[1], substitute_refs(node[2], fn))
    if tag in ("mod", "floordiv", "ceildiv"):
        return (tag, substitute_refs(node[1], fn), node[2])
    return node


# ---------------------------------------------------------------------------
# Maps and sets
# ---------------------------------------------------------------------------

def _strip_wrapper(text: str, keyword: str) -> str:
    t = text.strip()
    if t.startswith(keyword):
        rest = t[len(keyword):].strip()
        if not (rest.startswith("<") and rest.endswith(">")):
            raise ValueError(f"malformed {keyword}: {text!r}")
        return rest[1:-1]
    return t


@dataclass(frozen=True)
class AffineMap:
    n_dims: int
    exprs: Tuple[Expr, ...]
    source: str = field(default="", compare=False)
    n_syms: int = 0

    def eval(self, dims: Sequence[Any], syms: Sequence[Any] = ()) -> Tuple[Any, ...]:
        if len(dims) != self.n_dims:
            raise ValueError(f"affine map expects {self.n_dims} dims, got {len(dims)}: {self.source}")
        return tuple(eval_expr(e, dims, syms) for e in self.exprs)

    def _pure_dim(self, e: Expr) -> Optional[int]:
        lin = linearize(e, self.n_dims, self.n_syms)
        if lin is None:
            return None
        dc, sc, c = lin
        nz = [i for i, k in enumerate(dc) if k]
        if c or any(sc) or len(nz) != 1 or dc[nz[0]] != 1:
            return None
        return nz[0]

    def is_identity(self) -> bool:
        return len(self.exprs) == self.n_dims and all(
            self._pure_dim(e) == i for i, e in enumerate(self.exprs))

    def is_permutation(self) -> bool:
        if len(self.exprs) != self.n_dims:
            return False
        idx = [self._pure_dim(e) for e in self.exprs]
        return None not in idx and sorted(idx) == list(range(self.n_dims))

    def permutation(self) -> Optional[Tuple[int, ...]]:
        return tuple(self._pure_dim(e) for e in self.exprs) if self.is_permutation() else None


def parse_affine_map(text: str) -> AffineMap:
    inner = _strip_wrapper(text, "affine_map")
    toks = tokenize(inner)
    p = _ExprParser(toks)
    dims = p.ident_list("(", ")")
    syms: List[str] = []
    if p.peek() == "[":
        syms = p.ident_list("[", "]")
    p.dims = {n: i for i, n in enumerate(dims)}
    p.syms = {n: i for i, n in enumerate(syms)}
    p.take("->")
    p.take("(")
    exprs: List[Expr] = []
    while p.peek() != ")":
        exprs.append(p.expr())
        if p.peek() == ",":
            p.take(",")
    p.take(")")
    return AffineMap(len(dims), tuple(exprs), text.strip(), len(syms))


@dataclass(frozen=True)
class AffineSet:
    """Integer set; constraints are ("ge", expr) meaning expr >= 0 or ("eq", expr) meaning expr == 0."""
    n_dims: int
    constraints: Tuple[Tuple[str, Expr], ...]
    source: str = field(default="", compare=False)
    n_syms: int = 0

    def _mask(self, pts: Sequence[Any], syms: Sequence[Any] = ()):
        ok = True
        for kind, e in self.constraints:
            v = eval_expr(e, pts, syms)
            ok = ok & ((v == 0) if kind == "eq" else (v >= 0))
        return ok

    def contains(self, point: Sequence[int], syms: Sequence[int] = ()) -> bool:
        if len(point) != self.n_dims:
            return False
        return bool(self._mask(list(point), syms))

    def enumerate_array(self, shape: Tuple[int, ...], syms: Sequence[int] = ()) -> np.ndarray:
        """All points of the set inside [0, shape), row-major, as an (N, ndim) int64 array."""
        if len(shape) != self.n_dims:
            raise ValueError(f"affine set has {self.n_dims} dims, shape has {len(shape)}")
        grids = np.indices(tuple(int(s) for s in shape), dtype=np.int64).reshape(self.n_dims, -1)
        mask = self._mask(list(grids), syms)
        if mask is True:
            return grids.T.copy()
        return grids[:, np.asarray(mask, dtype=bool)].T.copy()

    def enumerate(self, shape: Tuple[int, ...], syms: Sequence[int] = ()) -> List[Tuple[int, ...]]:
        return [tuple(int(v) for v in p) for p in self.enumerate_array(shape, syms)]

    def is_full(self, shape: Tuple[int, ...]) -> bool:
        return len(self.enumerate_array(shape)) == int(np.prod(shape))


Bound = Any  # int or an Expr over symbols


def eval_bound(b: Bound, syms: Sequence[int]) -> int:
    return b if isinstance(b, int) else int(eval_expr(b, (), syms))


@dataclass(frozen=True)
class BoxSet:
    """Axis-aligned box {p : lo[d] <= p[d] < hi[d]} (bounds may be symbolic)."""
    lo: Tuple[Bound, ...]
    hi: Tuple[Bound, ...]

    @property
    def n_dims(self) -> int:
        return len(self.lo)

    @property
    def is_concrete(self) -> bool:
        return all(isinstance(b, int) for b in self.lo + self.hi)

    def specialize(self, syms: Sequence[int]) -> "BoxSet":
        return BoxSet(tuple(eval_bound(b, syms) for b in self.lo),
                      tuple(eval_bound(b, syms) for b in self.hi))

    def contains(self, point: Sequence[int], syms: Sequence[int] = ()) -> bool:
        box = self if self.is_concrete else self.specialize(syms)
        return len(point) == box.n_dims and all(
            box.lo[d] <= point[d] < box.hi[d] for d in range(box.n_dims))

    def extent(self) -> Tuple[int, ...]:
        return tuple(max(0, h - l) for l, h in zip(self.lo, self.hi))

    def is_empty(self) -> bool:
        return any(h <= l for l, h in zip(self.lo, self.hi))

    def enumerate_array(self, shape: Optional[Tuple[int, ...]] = None,
                        syms: Sequence[int] = ()) -> np.ndarray:
        box = self if self.is_concrete else self.specialize(syms)
        if shape is not None:
            if len(shape) != box.n_dims:
                raise ValueError("box/shape rank mismatch")
            for d in range(box.n_dims):
                if box.hi[d] > shape[d]:
                    raise ValueError(
                        f"box hi[{d}]={box.hi[d]} exceeds the tile shape {shape[d]}")
        ext = box.extent()
        if 0 in ext:
            return np.zeros((0, box.n_dims), dtype=np.int64)
        g = np.indices(ext, dtype=np.int64).reshape(box.n_dims, -1)
        g += np.asarray(box.lo, dtype=np.int64)[:, None]
        return g.T.copy()

    def enumerate(self, shape=None, syms=()) -> List[Tuple[int, ...]]:
        return [tuple(int(v) for v in p) for p in self.enumerate_array(shape, syms)]

    def is_full(self, shape: Tuple[int, ...]) -> bool:
        return tuple(self.lo) == (0,) * len(shape) and tuple(self.hi) == tuple(shape)

    @staticmethod
    def from_affine_set(aset: AffineSet) -> Optional["BoxSet"]:
        """Lower an axis-aligned, unit-coefficient, doubly-bounded set to a box."""
        lo: List[Optional[Bound]] = [None] * aset.n_dims
        hi: List[Optional[Bound]] = [None] * aset.n_dims

        def sym_term(sc, c):
            if not any(sc):
                return c
            node: Expr = ("c", c)
            for j, k in enumerate(sc):
                if k:
                    node = ("+", node, ("*", k, ("s", j)))
            return node

        def neg(b):
            return -b if isinstance(b, int) else ("neg", b)

        def add1(b):
            return b + 1 if isinstance(b, int) else ("+", b, ("c", 1))

        def tighten(cur, new, pick):
            if cur is None:
                return new
            if isinstance(cur, int) and isinstance(new, int):
                return pick(cur, new)
            return None  # symbolic bounds on both sides of one axis: not a box

        for kind, e in aset.constraints:
            lin = linearize(e, aset.n_dims, aset.n_syms)
            if lin is None:
                return None
            dc, sc, c = lin
            nz = [i for i, k in enumerate(dc) if k]
            if len(nz) != 1 or abs(dc[nz[0]]) != 1:
                return None
            i, k = nz[0], dc[nz[0]]
            t = sym_term(sc, c)
            if kind == "eq":
                pin = neg(t) if k == 1 else t
                lo[i] = tighten(lo[i], pin, max)
                hi[i] = tighten(hi[i], add1(pin), min)
                if lo[i] is None or hi[i] is None:
                    return None
            elif k == 1:
                lo[i] = tighten(lo[i], neg(t), max)
                if lo[i] is None:
                    return None
            else:
                hi[i] = tighten(hi[i], add1(t), min)
                if hi[i] is None:
                    return None
        if any(b is None for b in lo + hi):
            return None
        if all(isinstance(b, int) for b in lo + hi) and any(l >= h for l, h in zip(lo, hi)):
            return None
        return BoxSet(tuple(lo), tuple(hi))


def parse_affine_set_raw(text: str) -> AffineSet:
    inner = _strip_wrapper(text, "affine_set")
    toks = tokenize(inner)
    p = _ExprParser(toks)
    dims = p.ident_list("(", ")")
    syms: List[str] = []
    if p.peek() == "[":
        syms = p.ident_list("[", "]")
    p.dims = {n: i for i, n in enumerate(dims)}
    p.syms = {n: i for i, n in enumerate(syms)}
    p.take(":")
    p.take("(")
    cons: List[Tuple[str, Expr]] = []
    while p.peek() != ")":
        lhs = p.expr()
        op = p.take()
        rhs = p.expr()
        if op == ">=":
            cons.append(("ge", ("-", lhs, rhs)))
        elif op == "<=":
            cons.append(("ge", ("-", rhs, lhs)))
        elif op == "==":
            cons.append(("eq", ("-", lhs, rhs)))
        else:
            raise ValueError(f"unsupported constraint operator {op!r}")
        if p.peek() == ",":
            p.take(",")
    p.take(")")
    return AffineSet(len(dims), tuple(cons), text.strip(), len(syms))


def parse_affine_set(text: str):
    """BoxSet when axis-aligned (the reference's parse-time lowering), else AffineSet."""
    aset = parse_affine_set_raw(text)
    box = BoxSet.from_affine_set(aset)
    return box if box is not None else aset


def product_points(shape: Sequence[int]) -> List[Tuple[int, ...]]:
    return list(itertools.product(*(range(s) for s in shape)))
