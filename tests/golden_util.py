"""Loading and comparing the committed golden fixtures."""

import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"), allow_pickle=False)
    inputs = {k[4:]: z[k] for k in z.files if k.startswith("in__")}
    outputs = {k[5:]: z[k] for k in z.files if k.startswith("out__")}
    for k, v in inputs.items():
        outputs.setdefault(k, v)
    tol = float(z["tol"])
    seed, reads = None, None
    if "seed_meta" in z.files:
        import json
        seed = [(sp, core, addr, z[f"seed__{i}"])
                for i, (sp, core, addr) in enumerate(json.loads(str(z["seed_meta"])))]
        reads = [tuple(r) for r in json.loads(str(z["reads_meta"]))]
    return {
        "src": str(z["src"]), "func": str(z["func"]), "inputs": inputs, "outputs": outputs,
        "tol": None if tol < 0 else tol, "error": str(z["error"]),
        "error_msg": str(z["error_msg"]) if "error_msg" in z.files else "",
        "seed": seed, "reads": reads,
    }


def run_seeded(interp, g):
    """Run a golden case whose memory is seeded at fixed addresses (HBM sticks,
    LX bytes) through the `_prepare_execution` hook, as the reference's own
    tests do; returns the regions named by the case, read back after the call."""
    orig = interp._prepare_execution

    def prep(grid):
        orig(grid)
        for sp, core, addr, arr in g["seed"]:
            mem = interp.memory.hbm if sp == "HBM" else interp.memory.get_lx(core)
            mem.write(addr, arr.copy())
    interp._prepare_execution = prep
    interp.execute_function(g["func"], **{k: (v.copy() if isinstance(v, np.ndarray) else v)
                                          for k, v in g["inputs"].items()})
    out = {}
    for name, sp, core, addr, n, dt in g["reads"]:
        mem = interp.memory.hbm if sp == "HBM" else interp.memory.get_lx(core)
        out[name] = mem.read(addr, n, dt)
    return out


def run_seeded_oracle(oracle, g):
    """run_seeded for the oracle, which holds HBM only: the seeds are written
    into its HBM before the call.  Returns None for a case with memory in a
    core's LX."""
    if any(sp != "HBM" for sp, *_ in g["seed"]) or "spyre_memory_space<LX>" in g["src"]:
        return None
    oracle.preload = [(addr, arr) for _, _, addr, arr in g["seed"]]
    oracle.execute_function(g["func"], **{k: (v.copy() if isinstance(v, np.ndarray) else v)
                                          for k, v in g["inputs"].items()})
    return {name: oracle.hbm.read(addr, n, dt) for name, _, _, addr, n, dt in g["reads"]}


# smallest normal f16 (2^-14): relative errors are taken against at least this
# magnitude, so an output in the subnormal range is judged by its absolute error
# against that bound (one subnormal f16 step is about 1e-3 of it)
F16_TINY = 6.103515625e-05


def max_rel_err(got, want, floor=F16_TINY):
    got = got.astype(np.float64)
    want = want.astype(np.float64)
    denom = np.maximum(np.abs(want), floor)
    return float(np.max(np.abs(got - want) / denom)) if want.size else 0.0


def f16_ulp_distance(got, want):
    """Largest distance in f16 steps (units in the last place) between two arrays
    once both are rounded to f16; +0 and -0 are one value."""
    def ordered(x):
        b = np.asarray(x, np.float16).view(np.uint16).astype(np.int64)
        return np.where(b & 0x8000, 0x8000 - b, b)   # sign-magnitude -> ordered integers
    if want.size == 0:
        return 0
    return int(np.max(np.abs(ordered(got) - ordered(want))))


def err_report(got, want, tol=1e-2, floor=F16_TINY):
    """(max rel err, number of outputs above tol, max f16 ULP distance)."""
    g = got.astype(np.float64)
    w = want.astype(np.float64)
    rel = np.abs(g - w) / np.maximum(np.abs(w), floor)
    return (float(rel.max()) if rel.size else 0.0, int((rel > tol).sum()),
            f16_ulp_distance(got, want))


def assert_matches(name, got, want, tol):
    assert got.shape == want.shape and got.dtype == want.dtype, (name, got.shape, want.shape)
    if tol is None:
        if not np.array_equal(got, want, equal_nan=True):
            bad = np.argwhere(~((got == want) | (np.isnan(got.astype(np.float64)) &
                                                  np.isnan(want.astype(np.float64)))))
            raise AssertionError(f"{name}: not bit-exact at {len(bad)} positions, first {bad[:3].tolist()}")
    else:
        # max relative error over every output, |got - want| / max(|want|, 2^-14)
        err, n_bad, ulp = err_report(got, want, tol)
        print(f"{name}: max rel err {err:.3e}, max {ulp} f16 ulp")
        assert err <= tol, f"{name}: max rel err {err:.3e} > {tol} at {n_bad} outputs"


# unit roundoff of f32
U32 = 2.0 ** -24


def assert_contraction(name, got, want, mag, tol=1e-2, c=8.0, u=None):
    """Parity rule for f16 outputs of an f32-accumulated contraction (matmul,
    attention) against a reference computed exactly (float64) or by another f32
    order of accumulation.

    Every output must satisfy |got - want| <= tol * max(|want|, 2^-14) + c * u * mag,
    u = 2^-24 and mag = sum_k |a_k * b_k| for that output: the second term is
    the rounding noise of an f32 accumulation (any order of the sum carries
    about u * mag of it), so it only matters for outputs whose value cancels to
    below ~1e-4 of their terms, which no f32 implementation -- the reference's
    NumPy/OpenBLAS one included -- reproduces to 1e-2 relative.  The true max
    relative error (no noise term) and the number of outputs above tol are
    reported beside it; returns (max rel err, count above tol, max f16 ulp).
    For sums of f16-rounded block products the noise is that of f16 (u = 2^-11)
    times the sum of the block products' magnitudes."""
    g = got.astype(np.float64)
    w = want.astype(np.float64)
    err = np.abs(g - w)
    bound = tol * np.maximum(np.abs(w), F16_TINY) + c * (U32 if u is None else u) * \
        mag.astype(np.float64)
    rel, n_bad, ulp = err_report(got, want, tol)
    worst = float(np.max(err / bound)) if err.size else 0.0
    print(f"{name}: max rel err {rel:.3e} ({n_bad} of {w.size} outputs above {tol}), "
          f"max {ulp} f16 ulp, max err / bound {worst:.3f}")
    assert worst <= 1.0, (f"{name}: {int((err > bound).sum())} outputs outside "
                          f"tol * max(|w|, 2^-14) + {c} u sum|ab| (max rel err {rel:.3e})")
    return rel, n_bad, ulp


def attention_exact(q, k, v, heads, seq, scale, causal=True, group=8):
    """float64 attention on the GPU for [heads * seq, d] f16 torch tensors (host
    or device), rounded to f16, and the noise magnitude per output for
    assert_contraction: sum_j p_ij (1 + scale * sum_d |q k|) |v_j|, the value
    terms weighted by the logit's own f32 rounding noise.  Returns NumPy arrays."""
    import torch
    d = q.shape[1]
    out = torch.empty(heads * seq, d, dtype=torch.float16)
    mag = torch.empty(heads * seq, d, dtype=torch.float32)
    mask = torch.triu(torch.ones(seq, seq, dtype=torch.bool, device="cuda"), diagonal=1)
    for h0 in range(0, heads, group):
        n = min(group, heads - h0)
        sl = slice(h0 * seq, (h0 + n) * seq)
        qh = q[sl].cuda().double().view(n, seq, d)
        kh = k[sl].cuda().double().view(n, seq, d)
        vh = v[sl].cuda().double().view(n, seq, d)
        s = (qh @ kh.transpose(1, 2)) * scale
        if causal:
            s = s.masked_fill(mask, float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[sl] = (p @ vh).reshape(-1, d).half().cpu()
        sabs = (qh.abs() @ kh.abs().transpose(1, 2)) * scale
        mag[sl] = ((p * (1.0 + sabs)) @ vh.abs()).reshape(-1, d).float().cpu()
        del s, p, sabs
    return out.numpy(), mag.numpy()


def contraction_mag(name, inputs):
    """sum |terms| per output (the magnitude assert_contraction weighs the f32
    noise by) for the GEMM and attention workload cases, by case name
    ("gemm_...", "attention_..._seq<S>_..."), computed in float64 with NumPy;
    None for other cases."""
    import re
    if name.startswith("gemm"):
        a = np.abs(inputs["a_ptr"].astype(np.float64))
        b = np.abs(inputs["b_ptr"].astype(np.float64))
        return {"c_ptr": a @ b}
    if name.startswith("attention"):
        seq = int(re.search(r"seq(\d+)", name).group(1))
        d = inputs["q_ptr"].shape[1]
        scale = float(np.float16(1.0 / np.sqrt(d)))
        q, k, v = (inputs[n].astype(np.float64).reshape(-1, seq, d) for n in ("q_ptr", "k_ptr", "v_ptr"))
        s = np.einsum("hqd,hkd->hqk", q, k) * scale
        s = np.where(np.triu(np.ones((seq, seq), bool), 1), -np.inf, s)
        e = np.exp(s - s.max(-1, keepdims=True))
        pr = e / e.sum(-1, keepdims=True)
        sabs = np.einsum("hqd,hkd->hqk", np.abs(q), np.abs(k)) * scale
        return {"o_ptr": np.einsum("hqk,hkd->hqd", pr * (1 + sabs), np.abs(v)).reshape(-1, d)}
    return None


EXAMPLE_DIR = os.path.join(GOLDEN_DIR, "examples")


def example_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(EXAMPLE_DIR, "*.npz")))


def load_example(name):
    """A recorded reference example: its source, function, regenerated inputs
    (and memory seeds), and the reference's outputs, digests or exception."""
    import json
    import sys
    if GOLDEN_DIR not in sys.path:
        sys.path.insert(0, GOLDEN_DIR)
    import examples as E
    ex = E.BY_NAME[name]
    z = np.load(os.path.join(EXAMPLE_DIR, name + ".npz"), allow_pickle=False)
    tol = float(z["tol"])
    return {"src": str(z["src"]), "func": str(z["func"]), "inputs": E.inputs(ex),
            "seed": E.seeds(ex), "reads": ex["reads"], "tol": None if tol < 0 else tol,
            "error": str(z["error"]),
            "outputs": {k[5:]: z[k] for k in z.files if k.startswith("out__")},
            "digests": {k[8:]: json.loads(str(z[k])) for k in z.files if k.startswith("digest__")}}


def digest_of(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def example_mag(name, inputs):
    """({output: magnitude}, u) for the examples whose outputs are matmul
    results: they multiply f16 tiles, so each K block's product is rounded to
    f16 (u = 2^-11) and the magnitude is the sum over blocks of |A_blk @ B_blk|."""
    if "matmul" not in name:
        return {}, None
    a = inputs["a_ptr"].astype(np.float64)
    b = inputs["b_ptr"].astype(np.float64)
    bk = int(inputs["BLOCK_SIZE_K"])
    mag = np.zeros((a.shape[0], b.shape[1]))
    for k0 in range(0, a.shape[1], bk):
        mag += np.abs(a[:, k0:k0 + bk] @ b[k0:k0 + bk])
    return {"c_ptr": mag}, 2.0 ** -11
