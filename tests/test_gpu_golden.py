"""B200 parity: every golden fixture recorded from the reference, replayed on the GPU."""

import numpy as np
import pytest

from golden_util import (assert_contraction, assert_matches, contraction_mag, golden_names,
                         load_golden, run_seeded)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names())
def test_b200_matches_reference(name):
    from ktir_cpu_b200 import KTIRInterpreter
    g = load_golden(name)
    interp = KTIRInterpreter()
    interp.load(g["src"])
    if g["seed"] is not None:
        out = run_seeded(interp, g)
        for k, want in g["outputs"].items():
            assert_matches(f"{name}:{k}", out[k], want, g["tol"])
        return
    kw = {k: v.copy() for k, v in g["inputs"].items()}
    if g["error"]:
        with pytest.raises(Exception) as ei:
            interp.execute_function(g["func"], **kw)
        assert type(ei.value).__name__ == g["error"]
        return
    out = interp.execute_function(g["func"], **kw)
    _compare(name, g, out)


def _compare(name, g, out):
    """Bit-exact unless the case records a tolerance (exp/tanh/matmul results,
    where CUDA's f32 math and NumPy's differ by ulps); outputs of the GEMM and
    attention workloads are contractions, judged with their f32 noise."""
    mags = contraction_mag(name, g["inputs"]) or {}
    for k, want in g["outputs"].items():
        if k in mags and g["tol"] is not None:
            assert_contraction(f"{name}:{k}", out[k], want, mags[k], g["tol"])
        else:
            assert_matches(f"{name}:{k}", out[k], want, g["tol"])


def test_replay_uses_cached_plan():
    """A second call with the same signature reuses the traced plan."""
    from ktir_cpu_b200 import KTIRInterpreter
    g = load_golden("vector_add_n1024_grid8")
    interp = KTIRInterpreter()
    interp.load(g["src"])
    a = interp.execute_function(g["func"], **{k: v.copy() for k, v in g["inputs"].items()})
    exe = interp.last_executable
    b = interp.execute_function(g["func"], **{k: v.copy() for k, v in g["inputs"].items()})
    assert interp.last_executable is exe
    for k in a:
        assert np.array_equal(a[k], b[k])


@pytest.mark.parametrize("name", ["softmax_rows128_cols1024_grid4_chunk32",
                                  "gather_add_dups",
                                  "attention_batch1_heads2_seq256_dim128_grid2_bq64_bk64"])
def test_latency_report_alongside_gpu_run(name):
    """With latency_config set, a GPU call leaves the reference's report behind."""
    import json
    import os
    from ktir_cpu_b200 import HardwareConfig, KTIRInterpreter
    gold = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "latency.json")))
    g = load_golden(name)
    interp = KTIRInterpreter(latency_config=HardwareConfig())
    interp.load(g["src"])
    out = interp.execute_function(g["func"], **{k: v.copy() for k, v in g["inputs"].items()})
    _compare(name, g, out)
    rep = interp.get_latency_report()
    assert rep.kernel_cycles == gold[name]["kernel_cycles"]
    for cid, w in gold[name]["cores"].items():
        assert rep.counters[int(cid)].total_bytes == w["total_bytes"]
