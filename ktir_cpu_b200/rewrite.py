"""IR rewrites applied before tracing (the attention rewrite lives here)."""

from __future__ import annotations

from typing import Any, Dict

from .ir import IRFunction


def attention_rewrites(func: IRFunction) -> Dict[int, Any]:
    """Map id(scf.for op) -> tracer handler for recognised attention loops."""
    return {}


def match_attention_plan(low, stores):
    return None
