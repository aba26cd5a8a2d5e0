"""Tensor-core programs: the GEMM and attention matchers (tcgen05 kernels)."""

from __future__ import annotations


def match_gemm(low, stores):
    return None


def match_attention(low, stores):
    return None
