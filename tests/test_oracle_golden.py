"""The CPU oracle reproduces every golden fixture recorded from the reference."""

import numpy as np
import pytest

from golden_util import assert_matches, golden_names, load_golden, run_seeded_oracle
from oracle.interp import OracleInterpreter


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference(name):
    g = load_golden(name)
    o = OracleInterpreter()
    o.load(g["src"])
    if g["seed"] is not None:
        # memory seeded at fixed addresses; views in a core's LX (which the
        # oracle does not hold) are checked on the GPU alone
        out = run_seeded_oracle(o, g)
        if out is None:
            pytest.skip("views in LX are checked on the GPU against the recorded outputs")
        for k, want in g["outputs"].items():
            assert_matches(f"{name}:{k}", out[k], want, None)
        return
    kw = {k: v.copy() for k, v in g["inputs"].items()}
    if g["error"]:
        with pytest.raises(Exception) as ei:
            o.execute_function(g["func"], **kw)
        assert type(ei.value).__name__ == g["error"]
        return
    out = o.execute_function(g["func"], **kw)
    for k, want in g["outputs"].items():
        # the oracle restates the reference numerics exactly, so even the
        # tolerance cases are expected bit-exact here
        assert_matches(f"{name}:{k}", out[k], want, None)
