"""Latency report parity with the ktir-cpu reference tracker (host only).

The fixture tests/golden/latency.json holds the reference's report for every
golden case (make_latency_golden.py).  The B200 backend derives its report
from the host trace; totals, per-category cycles and flops, bytes and the
sequence of charged ops must be identical — the same floating-point values,
accumulated in the same order.  Zero-cost entries are not compared: the
reference's tokenizer folds a bare terminator line (``scf.yield``,
``return``) that follows a result-less ``scf.for`` into that op, so its
trace lists fewer zero-cost entries than the source has ops.
"""

import json
import os

import numpy as np
import pytest

from ktir_cpu_b200 import HardwareConfig, KTIRInterpreter
from ktir_cpu_b200.latency import LatencyCategory, category, rect_sticks

from golden.cases import CASES

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "latency.json")))
BY_NAME = {c["name"]: c for c in CASES}


def _report(name, trace=True):
    c = BY_NAME[name]
    interp = KTIRInterpreter(latency_config=HardwareConfig(), trace_latency=trace)
    interp.load(c["src"])
    return interp.estimate_latency(c["func"], **{k: v.copy() for k, v in c["inputs"].items()})


@pytest.mark.parametrize("name", sorted(GOLD))
def test_latency_matches_reference(name):
    want = GOLD[name]
    rep = _report(name)
    assert rep.kernel_cycles == want["kernel_cycles"]
    assert rep.bottleneck == want["bottleneck"]
    assert sorted(str(c) for c in rep.counters) == sorted(want["cores"])
    for cid, w in want["cores"].items():
        k = rep.counters[int(cid)]
        assert k.compute_cycles == w["compute_cycles"]
        assert k.memory_cycles == w["memory_cycles"]
        assert k.comm_cycles == w["comm_cycles"]
        assert k.total_bytes == w["total_bytes"]
        assert k.flops_by_category == w["flops_by_category"]
        assert k.cycles_by_category == w["cycles_by_category"]
        charged = [[e.op_type, e.category, e.cycles] for e in k.trace if e.category != "zero"]
        assert charged == w["charged"]
    rf = rep.roofline()
    for key in ("arithmetic_intensity", "peak_bw_gb_s", "dominant_unit", "efficiency"):
        assert rf[key] == want["roofline"][key], key


def test_hardware_config_defaults_and_derived():
    cfg = HardwareConfig()
    assert (cfg.num_cores, cfg.clock_ghz, cfg.hbm_bandwidth_tb_s, cfg.ring_bandwidth_tb_s,
            cfg.simd_elements_per_cycle, cfg.systolic_flops_per_cycle,
            cfg.transcendental_penalty) == (32, 1.0, 1.0, 4.0, 64, 2 * 64 ** 3, 4)
    assert cfg.hbm_bytes_per_cycle_per_core == pytest.approx(31.25)
    assert cfg.ring_bytes_per_cycle == pytest.approx(4000.0)
    assert HardwareConfig(clock_ghz=2.0).hbm_bytes_per_cycle_per_core == pytest.approx(15.625)


def test_categories():
    assert category("arith.addf") == LatencyCategory.COMPUTE_FLOAT
    assert category("arith.cmpi") == "compute_float"
    assert category("arith.addi") == "compute_int"
    assert category("math.exp") == "compute_transcendental"
    assert category("linalg.matmul") == "compute_matmul"
    assert category("ktdp.store") == "memory"
    assert category("linalg.reduce") == "zero"
    assert category("arith.truncf") == "zero"


def test_rect_sticks():
    # contiguous run: sticks spanned, counting partial ones at both ends
    assert rect_sticks(0x10000, (64,), (1,), 2) == 1
    assert rect_sticks(0x10000 + 64, (64,), (1,), 2) == 2
    # strided rows of 16 f16 with a 1024-element pitch: one stick per row
    assert rect_sticks(0x10000, (8, 16), (1024, 1), 2) == 8
    # a column of f16: every element on its own stick
    assert rect_sticks(0x10000, (32, 1), (128, 1), 2) == 32
    assert rect_sticks(0x10000, (0, 4), (8, 1), 2) == 0


def test_config_scaling_and_disabled_report():
    c = BY_NAME["vector_add_n1024_grid8"]
    base = _report("vector_add_n1024_grid8", trace=False)
    interp = KTIRInterpreter(latency_config=HardwareConfig(hbm_bandwidth_tb_s=2.0))
    interp.load(c["src"])
    fast = interp.estimate_latency(c["func"], **c["inputs"])
    for cid in base.counters:
        assert fast.counters[cid].memory_cycles == pytest.approx(
            base.counters[cid].memory_cycles / 2)
        assert fast.counters[cid].trace is None
    plain = KTIRInterpreter()
    plain.load(c["src"])
    assert plain.get_latency_report() is None
    text = str(base)
    assert "KTIR Latency Estimation Report" in text and "Roofline Analysis" in text
    s = base.summary_dict()
    assert s["num_cores"] == 8 and len(s["per_core"]) == 8


def test_indirect_sticks_follow_index_values():
    # the same gather charges fewer data sticks when every index hits one row
    c = BY_NAME["indirect_gather_4x4"]
    inputs = {k: v.copy() for k, v in c["inputs"].items()}
    interp = KTIRInterpreter(latency_config=HardwareConfig())
    interp.load(c["src"])
    spread = interp.estimate_latency(c["func"], **inputs).counters[0].total_bytes
    idx_name = [k for k, v in inputs.items() if v.dtype == np.int32][0]
    inputs[idx_name][:] = 0
    same = interp.estimate_latency(c["func"], **inputs).counters[0].total_bytes
    assert same <= spread


def test_seeded_distributed_cases_trace_on_the_host():
    """Distributed / LX view programs trace (and get a latency report) without a GPU."""
    from golden_util import golden_names, load_golden
    for name in golden_names():
        g = load_golden(name)
        if g["seed"] is None:
            continue
        interp = KTIRInterpreter(latency_config=HardwareConfig())
        interp.load(g["src"])
        orig = interp._prepare_execution

        def prep(grid, _o=orig, _g=g, _i=interp):
            _o(grid)
            for sp, core, addr, arr in _g["seed"]:
                mem = _i.memory.hbm if sp == "HBM" else _i.memory.get_lx(core)
                mem.write(addr, arr.copy())
        interp._prepare_execution = prep
        rep = interp.estimate_latency(g["func"])
        assert rep.kernel_cycles >= 0
