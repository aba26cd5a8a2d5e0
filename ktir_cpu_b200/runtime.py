"""ctypes binding of libktir_b200.so plus device-memory plumbing.

The structures below mirror include/ktir_b200.h field for field.  PyTorch is
used only to own device memory and streams; all compute goes through the
library.  Loading fails loudly when the library is missing or no CUDA device
is visible — there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import os
import struct
from typing import Optional

import numpy as np

from . import build as _build

MAX_BUFFERS = 16
MAX_RANK = 6
MAX_VIEWS = 12
MAX_INSTR = 64
NREG = 12
ARENA_SLOT = MAX_BUFFERS - 1

F16, F32, I32, I64, BOOL, U32 = 0, 1, 2, 3, 4, 5
STATUS_NEGATIVE_INDEX = 1
STATUS_TIMEOUT = 2

_DT = {np.dtype(np.float16): F16, np.dtype(np.float32): F32, np.dtype(np.int32): I32,
       np.dtype(np.int64): I64, np.dtype(np.bool_): BOOL, np.dtype(np.uint32): U32}


def dtype_code(dt) -> int:
    dt = np.dtype(dt)
    if dt not in _DT:
        raise NotImplementedError(f"tile dtype {dt} is not supported on the B200 backend")
    return _DT[dt]


class KtirBuffers(C.Structure):
    _fields_ = [("base", C.c_void_p * MAX_BUFFERS), ("numel", C.c_int64 * MAX_BUFFERS)]


class KtirView(C.Structure):
    _fields_ = [("slot", C.c_int32), ("dtype", C.c_int32), ("unit_col", C.c_int32),
                ("pad", C.c_int32), ("off", C.c_int64), ("stride", C.c_int64 * MAX_RANK)]


class KtirInstr(C.Structure):
    _fields_ = [("op", C.c_uint8), ("dst", C.c_uint8), ("a", C.c_uint8), ("b", C.c_uint8),
                ("c", C.c_uint8), ("dt", C.c_uint8), ("aux", C.c_uint8), ("flags", C.c_uint8),
                ("imm", C.c_int64)]


class KtirEwProgram(C.Structure):
    _fields_ = [("rank", C.c_int32), ("n_views", C.c_int32), ("n_instr", C.c_int32),
                ("n_units", C.c_int32), ("unit_cols", C.c_int32), ("contiguous", C.c_int32),
                ("numel", C.c_int64), ("shape", C.c_int64 * MAX_RANK),
                ("view", KtirView * MAX_VIEWS), ("code", KtirInstr * MAX_INSTR)]


class KtirSoftmaxDesc(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("n_units", C.c_int32),
                ("unit_cols", C.c_int32), ("compute_f16", C.c_int32), ("pad", C.c_int32),
                ("in_", KtirView), ("out", KtirView)]


class KtirGatherRmwDesc(C.Structure):
    _fields_ = [("table_slot", C.c_int32), ("idx_slot", C.c_int32), ("idx_dtype", C.c_int32),
                ("n_units", C.c_int32), ("unit_len", C.c_int32), ("row_len", C.c_int32),
                ("table_off", C.c_int64), ("row_stride", C.c_int64), ("idx_off", C.c_int64),
                ("idx_unit_stride", C.c_int64), ("row_lo", C.c_int64), ("row_hi", C.c_int64),
                ("phases", C.c_int32), ("pad2", C.c_int32), ("f", KtirEwProgram)]


class KtirReduceDesc(C.Structure):
    _fields_ = [("combiner", C.c_int32), ("dt", C.c_int32), ("n_units", C.c_int32),
                ("pad", C.c_int32), ("outer", C.c_int64), ("n", C.c_int64), ("inner", C.c_int64),
                ("in_off", C.c_int64), ("out_off", C.c_int64), ("tmp_off", C.c_int64),
                ("unit_stride", C.c_int64), ("in_slot", C.c_int32), ("out_slot", C.c_int32)]


class KtirMatmulDesc(C.Structure):
    _fields_ = [("batch", C.c_int64), ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
                ("a", KtirView), ("b", KtirView), ("out", KtirView),
                ("n_units", C.c_int32), ("unit_cols", C.c_int32)]


class KtirOffsetsDesc(C.Structure):
    _fields_ = [("buf", KtirView), ("dense", KtirView), ("count", C.c_int64),
                ("n_units", C.c_int32), ("scatter", C.c_int32)]


class KtirIndirectDesc(C.Structure):
    _fields_ = [("buf", KtirView), ("dense", KtirView), ("count", C.c_int64),
                ("n_units", C.c_int32), ("n_ind", C.c_int32), ("scatter", C.c_int32),
                ("pad", C.c_int32), ("idx_slot", C.c_int32 * 4), ("idx_dtype", C.c_int32 * 4),
                ("stride", C.c_int64 * 4)]


class KtirGemmDesc(C.Structure):
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p),
                ("lda", C.c_int64), ("ldb", C.c_int64), ("ldc", C.c_int64),
                ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
                ("add_zero", C.c_int32), ("pad", C.c_int32), ("status", C.c_void_p)]


class KtirFmhaDesc(C.Structure):
    _fields_ = [("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("o", C.c_void_p),
                ("bh", C.c_int64), ("seq", C.c_int64), ("d", C.c_int64), ("scale", C.c_float),
                ("causal", C.c_int32), ("row_stride", C.c_int64), ("status", C.c_void_p)]


class KtirGemmBlockedDesc(C.Structure):
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p),
                ("lda", C.c_int64), ("ldb", C.c_int64), ("ldc", C.c_int64),
                ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
                ("block_k", C.c_int32), ("acc_f16", C.c_int32), ("status", C.c_void_p)]


class KtirFmhaPartDesc(C.Structure):
    _fields_ = [("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("o", C.c_void_p),
                ("bh", C.c_int64), ("seq", C.c_int64), ("d", C.c_int64), ("kv_rows", C.c_int64),
                ("scale", C.c_float), ("causal", C.c_int32), ("n_qtiles", C.c_int32),
                ("kv_tiles", C.c_int32), ("key_mask", C.c_uint32), ("flags", C.c_int32),
                ("o_acc", C.c_void_p), ("ml", C.c_void_p), ("status", C.c_void_p),
                ("qtiles", C.c_uint8 * 32), ("kv_owner", C.c_uint8 * 32),
                ("kv_local", C.c_uint8 * 32)]


class KtirHostXfer(C.Structure):
    _fields_ = [("host", C.c_void_p), ("pinned", C.c_void_p), ("device", C.c_void_p),
                ("bytes", C.c_int64)]


class KtirHostCopy(C.Structure):
    _fields_ = [("dst", C.c_void_p), ("src", C.c_void_p), ("bytes", C.c_int64)]


EXPORTS = ["ktir_version", "ktir_last_error", "ktir_device_count", "ktir_ew",
           "ktir_softmax_rows", "ktir_gather_rmw", "ktir_reduce", "ktir_matmul",
           "ktir_offsets", "ktir_indirect", "ktir_gemm_f16", "ktir_gemm_f16_blocked", "ktir_fmha_f16",
           "ktir_fmha_f16_part", "ktir_copy_blocks", "ktir_pack_kv", "ktir_bytes_delta",
           "ktir_wait_selftest", "ktir_host_threads", "ktir_host_upload", "ktir_host_download",
           "ktir_ipc_alloc", "ktir_ipc_open", "ktir_ipc_close", "ktir_ipc_free", "ktir_flag_set",
           "ktir_flag_wait", "ktir_copy_async"]

_LIB: Optional[C.CDLL] = None


def lib_path() -> str:
    return _build.LIB


def load_library(build_if_missing: bool = False) -> C.CDLL:
    """Load libktir_b200.so (never falls back to anything else)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = lib_path()
    if not os.path.exists(path):
        if build_if_missing:
            _build.build()
        else:
            raise RuntimeError(
                f"{path} is missing: build it with `python -m ktir_cpu_b200.build`")
    lib = C.CDLL(path)
    vp, i32p, i64p = C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_int64)
    lib.ktir_version.restype = C.c_int
    lib.ktir_last_error.restype = C.c_char_p
    lib.ktir_device_count.argtypes = [i32p]
    lib.ktir_ew.argtypes = [C.POINTER(KtirEwProgram), C.POINTER(KtirBuffers), vp, vp]
    lib.ktir_softmax_rows.argtypes = [C.POINTER(KtirSoftmaxDesc), C.POINTER(KtirBuffers), vp, vp]
    lib.ktir_gather_rmw.argtypes = [C.POINTER(KtirGatherRmwDesc), C.POINTER(KtirBuffers), vp,
                                    C.c_int64, vp, vp]
    lib.ktir_reduce.argtypes = [C.POINTER(KtirReduceDesc), C.POINTER(KtirBuffers), vp]
    lib.ktir_matmul.argtypes = [C.POINTER(KtirMatmulDesc), C.POINTER(KtirBuffers), vp, vp]
    lib.ktir_offsets.argtypes = [C.POINTER(KtirOffsetsDesc), C.POINTER(KtirBuffers), vp, vp, vp]
    lib.ktir_indirect.argtypes = [C.POINTER(KtirIndirectDesc), C.POINTER(KtirBuffers), vp, vp,
                                  vp, vp, vp]
    lib.ktir_gemm_f16.argtypes = [C.POINTER(KtirGemmDesc), vp]
    lib.ktir_gemm_f16_blocked.argtypes = [C.POINTER(KtirGemmBlockedDesc), vp]
    lib.ktir_fmha_f16.argtypes = [C.POINTER(KtirFmhaDesc), vp]
    lib.ktir_fmha_f16_part.argtypes = [C.POINTER(KtirFmhaPartDesc), vp]
    lib.ktir_copy_blocks.argtypes = [vp, C.c_int64, vp, C.c_int64, C.c_int64, C.c_int64, vp]
    lib.ktir_bytes_delta.argtypes = [vp, vp, vp, C.c_int64, C.c_int32, vp]
    lib.ktir_pack_kv.argtypes = [vp, vp, vp, C.c_int64, C.c_int64, C.c_int64, C.c_uint32, vp]
    lib.ktir_wait_selftest.argtypes = [vp, C.c_uint32, vp]
    lib.ktir_ipc_alloc.argtypes = [C.c_int64, C.POINTER(vp), vp]
    lib.ktir_ipc_open.argtypes = [vp, C.POINTER(vp)]
    lib.ktir_ipc_close.argtypes = [vp]
    lib.ktir_ipc_free.argtypes = [vp]
    lib.ktir_flag_set.argtypes = [vp, C.c_uint32, vp]
    lib.ktir_flag_wait.argtypes = [vp, C.c_int32, C.c_int32, C.c_uint32, C.c_uint32, vp, vp]
    lib.ktir_copy_async.argtypes = [vp, vp, C.c_int64, vp]
    lib.ktir_host_threads.argtypes = []
    lib.ktir_host_upload.argtypes = [C.POINTER(KtirHostXfer), C.c_int, C.c_int, vp]
    lib.ktir_host_download.argtypes = [C.POINTER(KtirHostXfer), C.c_int, C.POINTER(KtirHostCopy),
                                       C.c_int, C.c_int, vp]
    for name in EXPORTS:
        getattr(lib, name).restype = C.c_int if name != "ktir_last_error" else C.c_char_p
    _LIB = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = _LIB.ktir_last_error().decode() if _LIB is not None else ""
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


def double_bits(v: float) -> int:
    return struct.unpack("<q", struct.pack("<d", float(v)))[0]


def require_cuda():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("the B200 backend needs a CUDA device; none is visible")
    return torch
