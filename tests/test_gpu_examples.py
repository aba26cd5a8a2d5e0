"""The reference's own example kernels on the B200, against the reference's
recorded results (tests/golden/examples): outputs bit-exact or within the
example's tolerance; outputs recorded as digests against the oracle run here
(test_oracle_examples.py pins the oracle to those digests); matmul outputs
under the contraction rule (golden_util.assert_contraction); the reference's
exception where it raised one.  Examples that address memory through
constants are seeded at those addresses through _prepare_execution, as the
reference's own tests do."""

import numpy as np
import pytest

from golden_util import (assert_contraction, assert_matches, example_mag, example_names,
                         load_example, run_seeded)
from oracle.interp import OracleInterpreter

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", example_names())
def test_b200_runs_reference_example(name):
    from ktir_cpu_b200 import KTIRInterpreter
    g = load_example(name)
    interp = KTIRInterpreter()
    interp.load(g["src"])
    kw = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in g["inputs"].items()}
    if g["error"]:
        with pytest.raises(Exception) as ei:
            interp.execute_function(g["func"], **kw)
        assert type(ei.value).__name__ == g["error"]
        return
    if g["seed"] is not None:
        out = run_seeded(interp, g)
    else:
        out = interp.execute_function(g["func"], **kw)
    mags, u = example_mag(name, g["inputs"])
    want = dict(g["outputs"])
    if g["digests"]:
        o = OracleInterpreter()
        o.load(g["src"])
        ref = o.execute_function(g["func"], **{k: (v.copy() if isinstance(v, np.ndarray) else v)
                                               for k, v in g["inputs"].items()})
        want.update({k: ref[k] for k in g["digests"]})
    for k, w in want.items():
        if k in mags and g["tol"] is not None:
            assert_contraction(f"{name}:{k}", out[k], w, mags[k], g["tol"], u=u)
        else:
            assert_matches(f"{name}:{k}", out[k], w, g["tol"])


# the examples whose plans must multiply on the tensor cores: the K-loop
# matmuls (tcgen05 GEMM plans) and the f16 products inside the 2-D SDPA
# (generic plan, ktir_gemm_f16_blocked per product)
TC_PLANS = {"ex_matmul_fwd": "gemm_blocked", "ex_matmul_small": "gemm_blocked",
            "ex_sdpa_2d": "matmul_tc"}


@pytest.mark.parametrize("name,kind", sorted(TC_PLANS.items()))
def test_example_matmuls_run_on_tensor_cores(name, kind):
    from ktir_cpu_b200 import KTIRInterpreter
    g = load_example(name)
    interp = KTIRInterpreter()
    interp.load(g["src"])
    interp.execute_function(g["func"], **{k: (v.copy() if isinstance(v, np.ndarray) else v)
                                          for k, v in g["inputs"].items()})
    kinds = [l.kind for l in interp.last_executable.plan.launches]
    assert kind in kinds, kinds
    assert "matmul" not in kinds, kinds
