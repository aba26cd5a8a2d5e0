"""The reference's own example kernels, as golden cases.

ktir-cpu ships example KTIR programs (examples/{triton-ktir,ktir,latency,rfc})
and its test fixture registry (tests/conftest.py:74-316) names, for each, the
scalar arguments it is executed with.  Each entry here gives the example's
path within the reference, its function, those scalar arguments, and how its
tensors are made: seeded NumPy arrays for the pointer arguments (shapes from
the example's memory views), or, for examples that address memory through
constants, the HBM sticks / LX bytes to seed before the call and the regions
to read after it.  make_examples.py runs the reference on every entry and
records the outcome; inputs are regenerated from the seeds here, so the
fixtures hold the example source, the outputs (or, for outputs above
OUTPUT_LIMIT bytes, digests) and any exception the reference raised.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, List

import numpy as np

OUTPUT_LIMIT = 1 << 20   # outputs above this many bytes are stored as digests


def _n(rng, shape, dtype=np.float16, scale=1.0):
    return (scale * rng.standard_normal(shape)).astype(dtype)


EXAMPLES: List[Dict[str, Any]] = []


def example(name, path, func, make: Callable[[np.random.Generator], Dict[str, Any]], tol=None,
            seed=None, reads=None, scalars=None):
    EXAMPLES.append({"name": name, "path": path, "func": func, "make": make, "tol": tol,
                     "seed_fn": seed, "reads": reads, "scalars": scalars or {}})


# --- triton-ktir ---------------------------------------------------------------------
example("ex_vector_add", "triton-ktir/vector_add_ktir.mlir", "add_kernel",
        lambda r: {"x_ptr": _n(r, 4096), "y_ptr": _n(r, 4096), "output_ptr": np.zeros(4096, np.float16)},
        scalars={"BLOCK_SIZE": 128})
for _ne in (256, 512, 1024):
    example(f"ex_vector_add_dynamic_n{_ne}", "triton-ktir/vector_add_dynamic_ktir.mlir",
            "add_kernel_dynamic",
            lambda r: {"x_ptr": _n(r, 1024, np.float32), "y_ptr": _n(r, 1024, np.float32),
                       "output_ptr": np.zeros(1024, np.float32)},
            scalars={"n_elements": _ne})
example("ex_softmax_fwd", "triton-ktir/softmax_fwd_ktir.mlir", "softmax_kernel",
        lambda r: {"output_ptr": np.zeros((4096, 1024), np.float16),
                   "input_ptr": _n(r, (4096, 1024), scale=2.0)},
        tol=1e-2, scalars={"n_rows": 4096})
example("ex_layernorm_fwd", "triton-ktir/layernorm_fwd_ktir.mlir", "_layer_norm_fwd_fused",
        lambda r: {"X": _n(r, (1151, 8192)), "Y": np.zeros((1151, 8192), np.float16),
                   "W": _n(r, (1151, 8192)), "B": _n(r, (1151, 8192)),
                   "Mean": np.zeros(1151, np.float16), "Rstd": np.zeros(1151, np.float16)},
        tol=1e-2, scalars={"N": 8192, "eps": 1e-5, "BLOCK_SIZE": 1024})
example("ex_matmul_fwd", "triton-ktir/matmul_fwd_ktir.mlir", "matmul_kernel",
        lambda r: {"a_ptr": r.uniform(-1, 1, (64, 2048)).astype(np.float16),
                   "b_ptr": r.uniform(-1, 1, (2048, 8192)).astype(np.float16),
                   "c_ptr": np.zeros((64, 8192), np.float16)},
        tol=1e-2, scalars={"K": 2048, "BLOCK_SIZE_M": 32, "BLOCK_SIZE_N": 512, "BLOCK_SIZE_K": 128})
example("ex_sdpa_2d", "triton-ktir/sdpa_2d.mlir", "sdpa_kernel_2d",
        lambda r: {"q_ptr": _n(r, (32, 64)), "k_ptr": _n(r, (32, 64)), "v_ptr": _n(r, (32, 64)),
                   "output_ptr": np.zeros((32, 64), np.float16)}, tol=1e-2)
example("ex_indexed_add", "triton-ktir/indexed_add.mlir", "indexed_add_kernel",
        lambda r: {"x_ptr": _n(r, (128, 64, 8, 128)), "y_ptr": _n(r, (2, 32, 8, 128)),
                   "index_ptr": r.choice(128, 2, replace=False).astype(np.int64),
                   "output_ptr": np.zeros((2, 32, 8, 128), np.float16)},
        scalars={"dim1_start": 0})
example("ex_paged_attention", "triton-ktir/paged_attention.mlir", "kernel_unified_attention_spyre_2d",
        lambda r: {"output_ptr": np.zeros((8, 32, 128), np.float16),
                   "query_ptr": _n(r, (8, 32, 128)),
                   "key_cache_ptr": _n(r, (64, 16, 8, 128)),
                   "value_cache_ptr": _n(r, (64, 16, 8, 128)),
                   "block_tables_ptr": r.permutation(64)[:16].astype(np.int32).reshape(1, 16)},
        tol=1e-2, scalars={"cur_batch_start_index": 0, "block_table_offset": 0, "num_tiles": 8,
                           "context_len": 120, "scale": 0.08838834764831843})

# --- latency ---------------------------------------------------------------------------
example("ex_softmax_small", "latency/softmax_small.mlir", "softmax_kernel_small",
        lambda r: {"output_ptr": np.zeros((64, 64), np.float16), "input_ptr": _n(r, (64, 64), scale=2.0)},
        tol=1e-2, scalars={"n_rows": 64})
example("ex_softmax_small_explicit", "latency/softmax_small_explicit.mlir",
        "softmax_kernel_small_explicit",
        lambda r: {"output_ptr": np.zeros((64, 64), np.float16), "input_ptr": _n(r, (64, 64), scale=2.0)},
        tol=1e-2, scalars={"n_rows": 64})
example("ex_matmul_small", "latency/matmul_small.mlir", "matmul_kernel_small",
        lambda r: {"a_ptr": r.uniform(-1, 1, (16, 64)).astype(np.float16),
                   "b_ptr": r.uniform(-1, 1, (64, 64)).astype(np.float16),
                   "c_ptr": np.zeros((16, 64), np.float16)},
        tol=1e-2, scalars={"K": 64, "BLOCK_SIZE_M": 8, "BLOCK_SIZE_N": 32, "BLOCK_SIZE_K": 32})
# 16 input rows of 128 f16 at sticks 0..31, 4 output rows at sticks 32..39
example("ex_ring_reduce_multi_group", "latency/ring_reduce_multi_group.mlir",
        "ring_reduce_multi_group", lambda r: {},
        seed=lambda r: [("HBM", 0, 0, _n(r, (16, 128))), ("HBM", 0, 32, np.zeros((4, 128), np.float16))],
        reads=[("out", "HBM", 0, 32, 512, "f16")], scalars={"in_ptr": 0, "out_ptr": 32})

# --- ktir ------------------------------------------------------------------------------
example("ex_reduce_generic", "ktir/reduce_generic.mlir", "reduce_explicit_region",
        lambda r: {"arg0": _n(r, (1, 4))})
example("ex_reduce_multiop", "ktir/reduce_multiop.mlir", "reduce_multiop",
        lambda r: {"arg0": _n(r, (1, 8))})
# 4 input rows of 128 f16 at sticks 0..7, the output row at sticks 8..9
example("ex_ring_reduce", "ktir/ring_reduce.mlir", "ring_reduce", lambda r: {},
        seed=lambda r: [("HBM", 0, 0, _n(r, (4, 128))), ("HBM", 0, 8, np.zeros(128, np.float16))],
        reads=[("out", "HBM", 0, 8, 128, "f16")], scalars={"in_ptr": 0, "out_ptr": 8})
example("ex_softmax_wide", "ktir/softmax_wide.mlir", "softmax_kernel",
        lambda r: {"output_ptr": np.zeros((2, 262144), np.float16),
                   "input_ptr": np.zeros((2, 262144), np.float16)})

# --- rfc (memory addressed through constants: seeded at those sticks / LX bytes) ------
example("ex_rfc_add_control_flow", "rfc/add-with-control-flow.mlir", "add", lambda r: {},
        seed=lambda r: [("HBM", 0, 1024, _n(r, (96, 64))), ("HBM", 0, 12288, _n(r, (96, 64))),
                        ("HBM", 0, 18432, np.zeros((96, 64), np.float16))],
        reads=[("C", "HBM", 0, 18432, 96 * 64, "f16")])
# rfc/distributed-view-copy.mlir is left out: its header notes that the
# reference resolves every <LX, core = N> view to the executing core's own
# scratchpad (its test is an expected failure), so its output depends on
# which core ran last and what that core's scratchpad held; the distributed
# and LX views are covered by the dist_* golden cases instead.
example("ex_rfc_indirect_access_copy", "rfc/indirect-access-copy.mlir", "indirect_access_copy",
        lambda r: {},
        seed=lambda r: [("HBM", 0, 0, _n(r, (64, 64))),
                        ("HBM", 0, 64, r.integers(0, 64, (64, 64)).astype(np.int32)),
                        ("HBM", 0, 128, r.integers(0, 64, (64, 64)).astype(np.int32)),
                        ("HBM", 0, 192, np.zeros((64, 64), np.float16))],
        reads=[("Y", "HBM", 0, 192, 64 * 64, "f16")])
example("ex_rfc_indirect_scatter", "rfc/indirect-scatter.mlir", "indirect_scatter",
        lambda r: {},
        seed=lambda r: [("HBM", 0, 0, _n(r, (64, 64))),
                        ("HBM", 0, 64, (_perm := r.permutation(64 * 64).reshape(64, 64).astype(np.int32)) // 64),
                        ("HBM", 0, 128, _perm % 64),
                        ("HBM", 0, 192, np.zeros((64, 64), np.float16))],
        reads=[("Y", "HBM", 0, 192, 64 * 64, "f16")])


def inputs(ex) -> Dict[str, Any]:
    """The example's keyword arguments: its tensors (seeded) and scalars."""
    rng = np.random.default_rng(_seed(ex["name"]))
    kw = dict(ex["make"](rng))
    kw.update(ex["scalars"])
    return kw


def seeds(ex):
    """The memory to seed before the call: (space, core, address, array) list."""
    if ex["seed_fn"] is None:
        return None
    return ex["seed_fn"](np.random.default_rng(_seed(ex["name"]) + 1))


def _seed(name: str) -> int:
    # a stable seed per example (Python's hash() of str is salted per process)
    return int.from_bytes(name.encode()[:8].ljust(8, b"\0"), "little") % (1 << 31)


BY_NAME = {e["name"]: e for e in EXAMPLES}
