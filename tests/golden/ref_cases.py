"""The cases behind tests/golden/ref_engine_c1.npz, shared by the script that runs the
reference's own engine and kernels (make_ref_engine_golden.py) and the tests that check the
CPU oracle against their outputs (test_ref_engine_golden.py).

Inputs come from a counter-based generator (splitmix64 of seed and index, mapped to
[-1, 1)), so the fixture stores only the outputs and both sides rebuild identical inputs.
"""
from __future__ import annotations

import numpy as np

# C1 tiny decode: the tiny configuration's 16-token prompt (ids uniform in [0, 4096),
# numpy default_rng(0).integers(0, 4096, 16), the engine tests' prompt, recorded here), 32 greedy
# steps, context 128
C1_PROMPT = [3484, 2608, 2093, 1105, 1260, 167, 308, 67, 717, 3331, 2660, 3738, 2062, 2484, 3976, 2988]
C1_GEN = 32
C1_CTX = 128
# steps whose full logits the fixture keeps (all steps keep their argmax token)
C1_KEEP = [0, 1, 7, 15, 16, 17, 23, 31, 39, 47]


def uniform(seed: int, n: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    """n float32 values in [lo, hi): splitmix64(seed * 2^32 + i) >> 40, scaled."""
    with np.errstate(over="ignore"):
        z = (np.arange(n, dtype=np.uint64) + np.uint64(seed) * np.uint64(1 << 32)) * np.uint64(0x9E3779B97F4A7C15)
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = (z >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    return (lo + (hi - lo) * u).astype(np.float32)


# Per-kernel cases: (kind, parameters). Matvec weights are tensors of the seeded synthetic
# models (source, tensor name); every vector is uniform(seed, n) scaled as written.
MATVEC = [
    # (case, shape name, weight type, tensor, x seed, x scale)
    ("q4_0_down", "tiny", 2, "blk.0.ffn_down.weight", 11, 1.0),
    ("q4_0_q", "tiny", 2, "blk.3.attn_q.weight", 12, 2.0),
    ("q4_k_gate", "k2", 12, "blk.1.ffn_gate.weight", 13, 1.0),
    ("q6_k_v", "k2", 12, "blk.0.attn_v.weight", 14, 1.5),
]
RMSNORM = [("n4096", 4096, 1e-5, 21, 3.0), ("n512", 512, 1e-5, 22, 0.5)]
ROPE = [("tiny_p77", 64, 8, 2, 77, 10000.0, 31), ("8b_p8191", 128, 32, 8, 8191, 500000.0, 32)]
ATTN = [("tiny_n100", 64, 8, 2, 100, 128, 41), ("8b_n520", 128, 32, 8, 520, 520, 42)]
SILU = [("n1408", 1408, 51, 4.0)]


def shapes():
    """The synthetic model shapes the matvec cases draw their weights from."""
    from types import SimpleNamespace as S
    tiny = S(n_layers=4, n_embd=512, n_heads=8, n_heads_kv=2, n_ff=1408, n_vocab=4096,
             rope_freq_base=10000.0, rms_norm_eps=1e-5, n_ctx_train=8192)
    k2 = S(n_layers=2, n_embd=512, n_heads=8, n_heads_kv=2, n_ff=1536, n_vocab=1024,
           rope_freq_base=10000.0, rms_norm_eps=1e-5, n_ctx_train=8192)
    return {"tiny": (tiny, 2, 0), "k2": (k2, 12, 14)}


def matvec_inputs(src, case):
    """(rows, cols, qtype, weight bytes, x) of a matvec case; `src(name)` gives a
    SynthSource-like object for the shape name."""
    _, sname, _, tensor, seed, scale = case
    s = src(sname)
    t, shp, _ = s.tensor_info(tensor)
    w = np.ascontiguousarray(s.read_rows(tensor))
    cols, rows = shp[0], shp[1]
    return rows, cols, t, w, uniform(seed, cols) * np.float32(scale)


def rmsnorm_inputs(case):
    _, n, eps, seed, scale = case
    return n, eps, uniform(seed, n) * np.float32(scale), uniform(seed + 1000, n, 0.5, 1.5)


def rope_inputs(case):
    _, hd, nh, nkv, pos, base, seed = case
    return hd, nh, nkv, pos, base, uniform(seed, nh * hd), uniform(seed + 1000, nkv * hd)


def attn_inputs(case):
    _, hd, nh, nkv, n_past, max_ctx, seed = case
    q = uniform(seed, nh * hd) * np.float32(2.0)
    kc = uniform(seed + 1000, max_ctx * nkv * hd)
    vc = uniform(seed + 2000, max_ctx * nkv * hd)
    return hd, nh, nkv, n_past, max_ctx, q, kc, vc


def silu_inputs(case):
    _, n, seed, scale = case
    return n, uniform(seed, n) * np.float32(scale), uniform(seed + 1000, n) * np.float32(scale)
