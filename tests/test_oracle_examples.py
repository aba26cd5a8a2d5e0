"""The oracle on the reference's own example kernels, against the reference's
recorded results (tests/golden/examples, made by make_examples.py): outputs
bit-exact, or within the tolerance the example records (exp / matmul), or,
for outputs recorded as digests, bit-identical bytes.  Examples that address
memory through constants are seeded at the same sticks first."""

import numpy as np
import pytest

from golden_util import assert_matches, digest_of, example_names, load_example, run_seeded_oracle
from oracle.interp import OracleInterpreter


@pytest.mark.parametrize("name", example_names())
def test_oracle_matches_reference_example(name):
    g = load_example(name)
    o = OracleInterpreter()
    o.load(g["src"])
    if g["seed"] is not None:
        out = run_seeded_oracle(o, g)
        if out is None:
            pytest.skip("views in LX are checked on the GPU against the recorded outputs")
        for k, want in g["outputs"].items():
            assert_matches(f"{name}:{k}", out[k], want, g["tol"])
        return
    kw = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in g["inputs"].items()}
    if g["error"]:
        with pytest.raises(Exception) as ei:
            o.execute_function(g["func"], **kw)
        assert type(ei.value).__name__ == g["error"]
        return
    out = o.execute_function(g["func"], **kw)
    for k, want in g["outputs"].items():
        assert_matches(f"{name}:{k}", out[k], want, g["tol"])
    for k, d in g["digests"].items():
        assert list(out[k].shape) == d["shape"] and str(out[k].dtype) == d["dtype"]
        assert digest_of(out[k]) == d["sha256"], f"{name}:{k} differs from the reference"
