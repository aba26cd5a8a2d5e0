"""Record tests/golden/examples/*.npz by running the ktir-cpu reference on its
own example kernels (the entries of examples.py).

Usage (REFERENCE_ROOT is a checkout of the ktir-cpu reference; the first
argument, else the KTIR_REFERENCE_ROOT environment variable):

    python tests/golden/make_examples.py REFERENCE_ROOT [NAME ...]

Each fixture holds the example's source text, its function and scalar
arguments, and either the exception the reference raised or its outputs:
every tensor argument the call changed, and every memory region the entry
names, in full up to OUTPUT_LIMIT bytes, above that as a digest (SHA-256 of
the bytes, float64 sum and sum of magnitudes).  Inputs are not stored: the
tests regenerate them from the seeds in examples.py.  Only this script
imports the reference.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "examples")


def digest(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    f = a.astype(np.float64)
    return json.dumps({"sha256": hashlib.sha256(a.tobytes()).hexdigest(), "shape": list(a.shape),
                       "dtype": str(a.dtype), "sum": float(np.nansum(f)),
                       "abs_sum": float(np.nansum(np.abs(f)))})


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KTIR_REFERENCE_ROOT")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "ktir_cpu")):
        raise SystemExit("give the reference checkout as the first argument "
                         "(or set KTIR_REFERENCE_ROOT)")
    only = set(sys.argv[2:])
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    sys.path.insert(0, HERE)
    import warnings
    warnings.filterwarnings("ignore")
    from ktir_cpu import KTIRInterpreter  # the reference
    import examples as E
    os.makedirs(OUT, exist_ok=True)
    for ex in E.EXAMPLES:
        if only and ex["name"] not in only:
            continue
        src = open(os.path.join(ref_root, "examples", ex["path"])).read()
        kw = E.inputs(ex)
        seeds = E.seeds(ex)
        interp = KTIRInterpreter()
        interp.load(src)
        rec = {"src": np.array(src), "func": np.array(ex["func"]), "path": np.array(ex["path"]),
               "scalars": np.array(json.dumps(ex["scalars"])),
               "tol": np.array(-1.0 if ex["tol"] is None else ex["tol"])}
        if seeds is not None:
            orig = interp._prepare_execution

            def prep(grid, _orig=orig, _seeds=seeds, _interp=interp):
                _orig(grid)
                for sp, core, addr, arr in _seeds:
                    mem = _interp.memory.hbm if sp == "HBM" else _interp.memory.get_lx(core)
                    mem.write(addr, arr.copy())
            interp._prepare_execution = prep
        t0 = time.time()
        outs = {}
        try:
            res = interp.execute_function(ex["func"], **{k: (v.copy() if isinstance(v, np.ndarray) else v)
                                                         for k, v in kw.items()})
            for k, v in res.items():
                if not np.array_equal(v, kw[k], equal_nan=True):
                    outs[k] = v
            for name, sp, core, addr, n, dt in ex["reads"] or []:
                mem = interp.memory.hbm if sp == "HBM" else interp.memory.get_lx(core)
                outs[name] = mem.read(addr, n, dt)
            rec["error"] = np.array("")
            status = "ok"
        except Exception as e:  # record what the reference raised
            rec["error"] = np.array(type(e).__name__)
            rec["error_msg"] = np.array(str(e))
            status = type(e).__name__
        for k, v in outs.items():
            if v.nbytes <= E.OUTPUT_LIMIT:
                rec["out__" + k] = v
            else:
                rec["digest__" + k] = np.array(digest(v))
        np.savez_compressed(os.path.join(OUT, ex["name"] + ".npz"), **rec)
        print(f"{ex['name']:36s} {status:14s} {time.time() - t0:8.2f}s  outputs {sorted(outs)}")


if __name__ == "__main__":
    main()
