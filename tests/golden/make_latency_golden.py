"""Regenerate tests/golden/latency.json from the ktir-cpu reference's latency tracker.

Usage (REFERENCE_ROOT is a checkout of the ktir-cpu reference; the first
argument, else the KTIR_REFERENCE_ROOT environment variable):

    python tests/golden/make_latency_golden.py REFERENCE_ROOT

Every case of ``cases.py`` that the reference executes without error is run
once with ``latency_config=HardwareConfig()`` and ``trace_latency=True``; the
fixture keeps, per core, the counters' totals and the charged (non-zero
category) trace entries in op order.  Only this script imports the reference.
"""

from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KTIR_REFERENCE_ROOT")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "ktir_cpu")):
        raise SystemExit("give the reference checkout as the first argument "
                         "(or set KTIR_REFERENCE_ROOT)")
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    sys.path.insert(0, REPO)
    sys.path.insert(0, HERE)
    import warnings
    warnings.filterwarnings("ignore")
    from ktir_cpu import KTIRInterpreter  # the reference
    from ktir_cpu.latency import HardwareConfig
    from cases import CASES

    out = {}
    for c in CASES:
        if c["expect_error"]:
            continue
        interp = KTIRInterpreter(latency_config=HardwareConfig(), trace_latency=True)
        interp.load(c["src"])
        if "seed" in c:
            # memory seeded at fixed addresses before the call, as for the
            # value fixtures (HBM sticks, LX bytes)
            orig = interp._prepare_execution

            def prep(grid, _orig=orig, _c=c, _interp=interp):
                _orig(grid)
                for sp, core, addr, arr in _c["seed"]:
                    mem = _interp.memory.hbm if sp == "HBM" else _interp.memory.get_lx(core)
                    mem.write(addr, arr.copy())
            interp._prepare_execution = prep
        try:
            interp.execute_function(c["func"], **{k: v.copy() for k, v in c["inputs"].items()})
        except AttributeError as e:
            # the reference tracker does not size distributed tile
            # references (DistributedTileRef has no memref): no fixture
            print(f"{c['name']:44s} skipped: {e}")
            continue
        rep = interp.get_latency_report()
        cores = {}
        for cid, k in sorted(rep.counters.items()):
            cores[str(cid)] = {
                "compute_cycles": k.compute_cycles, "memory_cycles": k.memory_cycles,
                "comm_cycles": k.comm_cycles, "total_bytes": k.total_bytes,
                "flops_by_category": k.flops_by_category,
                "cycles_by_category": k.cycles_by_category,
                "charged": [[e.op_type, str(e.category), e.cycles] for e in k.trace
                            if str(e.category) != "zero"],
            }
        out[c["name"]] = {"kernel_cycles": rep.kernel_cycles, "bottleneck": rep.bottleneck,
                          "roofline": rep.roofline(), "cores": cores}
        print(f"{c['name']:44s} {rep.kernel_cycles:14.3f} cycles")
    with open(os.path.join(HERE, "latency.json"), "w") as f:
        json.dump(out, f, indent=None, separators=(",", ":"))


if __name__ == "__main__":
    main()
