"""Regenerate tests/golden/*.npz by running the ktir-cpu reference interpreter.

Usage (REFERENCE_ROOT is a checkout of the ktir-cpu reference; the first
argument, else the KTIR_REFERENCE_ROOT environment variable):

    python tests/golden/make_golden.py REFERENCE_ROOT [CASE_NAME ...]

With case names, only those fixtures are regenerated.

For every case in ``cases.py`` it stores the KTIR source, function name,
inputs, and either the reference outputs or the name and message of the
exception the reference raised.  Only this script imports the reference;
the tests read the committed fixtures.
"""

from __future__ import annotations

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KTIR_REFERENCE_ROOT")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "ktir_cpu")):
        raise SystemExit("give the reference checkout as the first argument "
                         "(or set KTIR_REFERENCE_ROOT)")
    only = set(sys.argv[2:])
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    sys.path.insert(0, REPO)
    sys.path.insert(0, HERE)
    import warnings
    warnings.filterwarnings("ignore")
    from ktir_cpu import KTIRInterpreter  # the reference
    from cases import CASES

    for c in CASES:
        if only and c["name"] not in only:
            continue
        interp = KTIRInterpreter()
        interp.load(c["src"])
        kw = {k: v.copy() for k, v in c["inputs"].items()}
        rec = {"src": np.array(c["src"]), "func": np.array(c["func"]),
               "tol": np.array(-1.0 if c["tol"] is None else c["tol"])}
        for k, v in c["inputs"].items():
            rec["in__" + k] = v
        seeded = "seed" in c
        if seeded:
            # memory seeded at fixed addresses before the call (HBM sticks, LX
            # bytes) through the _prepare_execution hook, read back after it
            rec["seed_meta"] = np.array(json.dumps([[sp, core, addr] for sp, core, addr, _ in c["seed"]]))
            rec["reads_meta"] = np.array(json.dumps(c["reads"]))
            for i, (_, _, _, arr) in enumerate(c["seed"]):
                rec[f"seed__{i}"] = arr
            orig = interp._prepare_execution

            def prep(grid, _orig=orig, _c=c, _interp=interp):
                _orig(grid)
                for sp, core, addr, arr in _c["seed"]:
                    mem = _interp.memory.hbm if sp == "HBM" else _interp.memory.get_lx(core)
                    mem.write(addr, arr.copy())
            interp._prepare_execution = prep
        t0 = time.time()
        try:
            out = interp.execute_function(c["func"], **kw)
            if seeded:
                for name, sp, core, addr, n, dt in c["reads"]:
                    mem = interp.memory.hbm if sp == "HBM" else interp.memory.get_lx(core)
                    rec["out__" + name] = mem.read(addr, n, dt)
            for k, v in out.items():
                # unchanged buffers are not stored twice
                if not np.array_equal(v, c["inputs"][k], equal_nan=True):
                    rec["out__" + k] = v
            rec["error"] = np.array("")
            status = "ok"
        except Exception as e:  # record what the reference raised
            rec["error"] = np.array(type(e).__name__)
            rec["error_msg"] = np.array(str(e))
            status = type(e).__name__
        dt = time.time() - t0
        if c["expect_error"] and status != c["expect_error"]:
            raise SystemExit(f"{c['name']}: expected {c['expect_error']}, reference gave {status}")
        np.savez_compressed(os.path.join(HERE, c["name"] + ".npz"), **rec)
        print(f"{c['name']:44s} {status:12s} {dt:7.2f}s")


if __name__ == "__main__":
    main()
