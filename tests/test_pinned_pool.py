"""Host logic of the page-locked result pool (ktir_cpu_b200.interpreter._PinnedPool),
with ordinary CPU tensors standing in for page-locked ones: a buffer is handed
out again only once nothing refers to it (results, views of results), buffers
are kept per size, and a call that would grow the pool past its limit gets
nothing (it then stages through buffers of its own)."""

import gc

import numpy as np
import torch

from ktir_cpu_b200.interpreter import _PinnedPool


class _CpuTorch:
    uint8 = torch.uint8

    @staticmethod
    def empty(n, dtype, pin_memory):
        return torch.empty(n, dtype=dtype)


def _ptrs(staged):
    return [a.ctypes.data for _, a in staged]


def test_idle_buffers_are_reused_per_size():
    pool = _PinnedPool()
    first = _ptrs(pool.take([4096, 8192], _CpuTorch))
    gc.collect()
    again = _ptrs(pool.take([8192, 4096], _CpuTorch))
    assert sorted(first) == sorted(again)
    assert pool.bytes == 4096 + 8192


def test_held_results_and_views_keep_their_buffers():
    pool = _PinnedPool()
    staged = pool.take([4096], _CpuTorch)
    result = staged[0][1][:1000].view(np.uint16)      # what a call returns
    view = result[10:20]                              # a view the caller keeps
    del staged, result
    gc.collect()
    second = pool.take([4096], _CpuTorch)
    assert second[0][1].ctypes.data != view.ctypes.data - 20
    assert pool.bytes == 2 * 4096
    del second, view
    gc.collect()
    third = pool.take([4096, 4096], _CpuTorch)
    assert pool.bytes == 2 * 4096 and len(set(_ptrs(third))) == 2


def test_one_call_never_gets_the_same_buffer_twice():
    pool = _PinnedPool()
    staged = pool.take([4096, 4096, 4096], _CpuTorch)
    assert len(set(_ptrs(staged))) == 3


def test_limit_makes_the_call_fall_back():
    pool = _PinnedPool()
    pool.limit = 10000
    assert pool.take([8192], _CpuTorch) is not None
    gc.collect()
    assert pool.take([8192], _CpuTorch) is not None          # reuses the idle buffer
    held = pool.take([8192], _CpuTorch)
    assert pool.take([8192], _CpuTorch) is None               # would need a second 8 KiB
    assert pool.bytes == 8192
    del held
