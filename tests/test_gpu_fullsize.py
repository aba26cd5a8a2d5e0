"""Parity at the full benchmark sizes of the two tensor-core workloads.

GEMM f16 4096^3 on the 8x4 core grid and causal attention B4 H32 S2048 D128 on
32 cores run through KTIRInterpreter.execute_function.  Each is compared, over
the whole output, with the same computation done in float64 on the GPU and
rounded to f16, and, on a sample of cores, with the NumPy oracle of the
reference interpreter (the first cores of the grid; the oracle would take
minutes for the whole call).  The rule is the max relative error <= 1e-2 of
every f16 output (|got - want| / max(|want|, 2^-14)), plus, for outputs that
cancel to below the f32 rounding noise of their own sum, that noise
(golden_util.assert_contraction).
"""

import numpy as np
import pytest

from golden_util import assert_contraction, attention_exact
from ktir_cpu_b200 import workloads as W
from oracle.interp import OracleInterpreter

pytestmark = pytest.mark.gpu

ORACLE_CORES = 2


def _device_run(name):
    from ktir_cpu_b200 import KTIRInterpreter
    kw = W.inputs(name, seed=0)
    dev = KTIRInterpreter()
    dev.load(W.source(name))
    got = dev.execute_function(W.FUNC[name], **{k: v.copy() for k, v in kw.items()})
    return kw, got, dev


def _oracle_sample(name, kw, out_key):
    """The oracle on the first ORACLE_CORES cores; output elements those cores
    did not write stay NaN and are left out of the comparison."""
    ora = OracleInterpreter()
    ora.load(W.source(name))
    ora.core_limit = ORACLE_CORES
    args = {k: v.copy() for k, v in kw.items()}
    args[out_key] = np.full_like(kw[out_key], np.nan)
    want = ora.execute_function(W.FUNC[name], **args)[out_key]
    return want, ~np.isnan(want.astype(np.float32))


def test_gemm_full_size_c3():
    import torch
    kw, got, dev = _device_run("gemm")
    assert dev.last_executable.plan.kind == "gemm"
    a = torch.from_numpy(kw["a_ptr"]).cuda()
    b = torch.from_numpy(kw["b_ptr"]).cuda()
    exact = (a.double() @ b.double()).half().cpu().numpy()
    mag = (a.float().abs() @ b.float().abs()).cpu().numpy()   # sum_k |a b|, terms >= 0
    c = got["c_ptr"]
    assert np.isfinite(c.astype(np.float32)).all()
    assert_contraction("C3 gemm vs float64", c, exact, mag)
    want, cover = _oracle_sample("gemm", kw, "c_ptr")
    assert cover.sum() == ORACLE_CORES * 512 * 1024
    assert_contraction("C3 gemm vs oracle (2 cores)", c[cover], want[cover], mag[cover])
    # the oracle's own distance from the exact result, for the record
    assert_contraction("C3 oracle vs float64 (2 cores)", want[cover], exact[cover], mag[cover])


def test_attention_full_size_c5():
    import torch
    kw, got, dev = _device_run("attention")
    assert dev.last_executable.plan.kind == "attention"
    p = W.FULL["attention"]
    heads, seq = p["batch"] * p["heads"], p["seq"]
    scale = float(np.float16(1.0 / np.sqrt(p["dim"])))   # the f16-coerced scalar operand
    q, k, v = (torch.from_numpy(kw[n]) for n in ("q_ptr", "k_ptr", "v_ptr"))
    exact, mag = attention_exact(q, k, v, heads, seq, scale, causal=True)
    o = got["o_ptr"]
    assert np.isfinite(o.astype(np.float32)).all()
    assert_contraction("C5 attention vs float64", o, exact, mag)
    want, cover = _oracle_sample("attention", kw, "o_ptr")
    assert cover.sum() == ORACLE_CORES * (heads // p["grid"]) * seq * p["dim"]
    assert_contraction("C5 attention vs oracle (2 cores)", o[cover], want[cover], mag[cover])
    assert_contraction("C5 oracle vs float64 (2 cores)", want[cover], exact[cover], mag[cover])
