"""The C ABI: the library exports every declared entry point, and the ctypes
mirrors of the descriptor structs have the C layout (checked with gcc)."""

import ctypes as C
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ktir_b200.h")

STRUCTS = ["KtirBuffers", "KtirView", "KtirInstr", "KtirEwProgram", "KtirSoftmaxDesc",
           "KtirGatherRmwDesc", "KtirReduceDesc", "KtirMatmulDesc", "KtirOffsetsDesc",
           "KtirIndirectDesc", "KtirGemmDesc", "KtirGemmBlockedDesc", "KtirFmhaDesc", "KtirFmhaPartDesc", "KtirHostXfer",
           "KtirHostCopy"]


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ktir_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "ktir_ew" in names and "ktir_gemm_f16" in names and len(names) >= 12


def test_library_exports_every_declared_symbol():
    from ktir_cpu_b200 import runtime as R
    lib = C.CDLL(R.lib_path())
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_loads_without_a_gpu():
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    assert lib.ktir_version() >= 100


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_struct_layouts_match_the_header(tmp_path):
    from ktir_cpu_b200 import runtime as R
    src = tmp_path / "sizes.c"
    src.write_text('#include <stdio.h>\n#include "ktir_b200.h"\nint main(void){\n' +
                   "".join(f'printf("{s} %zu\\n", sizeof({s}));\n' for s in STRUCTS) + "return 0;}\n")
    exe = tmp_path / "sizes"
    subprocess.check_call(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)])
    out = subprocess.check_output([str(exe)]).decode().split()
    c_sizes = dict(zip(out[0::2], map(int, out[1::2])))
    for s in STRUCTS:
        assert C.sizeof(getattr(R, s)) == c_sizes[s], s


def test_host_staging_pool_and_loud_failure_without_a_gpu():
    """The staging worker pool starts without a GPU; a transfer then fails
    with an error code and a message instead of touching memory."""
    import numpy as np
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    assert lib.ktir_host_threads() >= 1
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("checks the behaviour without a GPU")
    except ImportError:
        pass
    a = np.arange(16, dtype=np.uint8)
    x = R.KtirHostXfer()
    x.host, x.pinned, x.device, x.bytes = a.ctypes.data, a.ctypes.data, a.ctypes.data, 16
    assert lib.ktir_host_upload(C.byref(x), 1, 0, None) < 0
    assert lib.ktir_last_error()
    assert lib.ktir_host_upload(None, -1, 0, None) < 0
