"""The CPU oracle against outputs of the reference's OWN engine and CUDA kernels
(tests/golden/ref_engine_c1.npz, made by tests/golden/make_ref_engine_golden.py on a GPU
from oracle/_ref/ref_engine: reference src/engine.cpp + cuda/*.cu compiled unmodified).

This pins the oracle's forward restatement (matvec, RMSNorm, RoPE, KV layout, attention,
SiLU, layer order, final norm, LM head, greedy argmax) to the reference's behaviour, so
that the B200 engine's parity tests against the oracle are parity against the reference.
CPU only: the fixture is committed.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import ref_cases as RC  # noqa: E402

FIX = os.path.join(HERE, "golden", "ref_engine_c1.npz")


@pytest.fixture(scope="module")
def fix():
    return np.load(FIX)


@pytest.fixture(scope="module")
def oracle_mod():
    from oracle import oracle
    return oracle


def rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(1e-30, np.max(np.abs(b))))


def run_oracle_c1(oracle, tokens, kv_f16):
    shp, _, _ = RC.shapes()["tiny"]
    src = oracle.SynthSource(shp, seed=0)
    om = oracle.OracleModel(src, max_ctx=RC.C1_CTX, kv_f16=kv_f16)
    logits = []
    for t in tokens:
        logits.append(om.forward(int(t)))
    om.close()
    return np.stack(logits)


def test_fixture_shape(fix):
    n = len(RC.C1_PROMPT) + RC.C1_GEN
    assert fix["c1_tokens"].shape == (n,)
    assert list(fix["c1_tokens"][:len(RC.C1_PROMPT)]) == RC.C1_PROMPT
    assert list(fix["c1_keep"]) == RC.C1_KEEP
    assert fix["c1_logits"].shape == (len(RC.C1_KEEP), 4096)


def test_oracle_decode_matches_reference_engine(fix, oracle_mod):
    """fp32 KV cache, as the reference keeps it: the oracle's logits equal the reference
    engine's to float rounding, and all 32 greedy tokens are the same."""
    toks = fix["c1_tokens"]
    lg = run_oracle_c1(oracle_mod, toks, kv_f16=False)
    np_ = len(RC.C1_PROMPT)
    for i, s in enumerate(RC.C1_KEEP):
        e = rel(lg[s], fix["c1_logits"][i])
        assert e < 1e-4, f"step {s}: logits relative error {e:.3g}"
    got = [oracle_mod.argmax(lg[s]) for s in range(np_ - 1, len(toks) - 1)]
    assert got == [int(t) for t in toks[np_:]]


def test_oracle_fp16_kv_within_logit_bar(fix, oracle_mod):
    """The fp16 KV cache of the B200 engine (the oracle's kv_f16 mode) stays within the 1e-2
    logits bar of the reference's fp32 cache and keeps every greedy token."""
    toks = fix["c1_tokens"]
    lg = run_oracle_c1(oracle_mod, toks, kv_f16=True)
    for i, s in enumerate(RC.C1_KEEP):
        assert rel(lg[s], fix["c1_logits"][i]) < 1e-2
    np_ = len(RC.C1_PROMPT)
    assert [oracle_mod.argmax(lg[s]) for s in range(np_ - 1, len(toks) - 1)] == [int(t) for t in toks[np_:]]


@pytest.mark.parametrize("case", RC.MATVEC, ids=lambda c: c[0])
def test_matvec_matches_reference_kernel(fix, oracle_mod, case):
    cache = {}

    def src(name):
        if name not in cache:
            shp, wt, mt = RC.shapes()[name]
            cache[name] = oracle_mod.SynthSource(shp, seed=0, weight_type=wt, mix_type=mt)
        return cache[name]
    rows, cols, qt, w, x = RC.matvec_inputs(src, case)
    y = oracle_mod.matvec(w, qt, x, rows, cols)
    assert rel(y, fix["matvec_" + case[0]]) < 1e-5


@pytest.mark.parametrize("case", RC.RMSNORM, ids=lambda c: c[0])
def test_rmsnorm_matches_reference_kernel(fix, oracle_mod, case):
    n, eps, x, w = RC.rmsnorm_inputs(case)
    assert rel(oracle_mod.rmsnorm(x, w, eps), fix["rmsnorm_" + case[0]]) < 1e-6


@pytest.mark.parametrize("case", RC.ROPE, ids=lambda c: c[0])
def test_rope_matches_reference_kernel(fix, oracle_mod, case):
    """Up to position 8191 with theta 5e5 (angles to ~8e3 rad), fp32 powf/cosf/sinf on both
    sides agree to float rounding."""
    hd, nh, nkv, pos, base, q, k = RC.rope_inputs(case)
    qo, ko = oracle_mod.rope(q, k, hd, nh, nkv, pos, base)
    assert rel(np.concatenate([qo, ko]), fix["rope_" + case[0]]) < 1e-5


@pytest.mark.parametrize("case", RC.ATTN, ids=lambda c: c[0])
def test_attention_matches_reference_kernel(fix, oracle_mod, case):
    hd, nh, nkv, n_past, max_ctx, q, kc, vc = RC.attn_inputs(case)
    out = oracle_mod.attention(q, kc[:n_past * nkv * hd], vc[:n_past * nkv * hd], hd, nh, nkv, n_past)
    assert rel(out, fix["attention_" + case[0]]) < 1e-5


@pytest.mark.parametrize("case", RC.SILU, ids=lambda c: c[0])
def test_silu_matches_reference_kernel(fix, oracle_mod, case):
    n, g, u = RC.silu_inputs(case)
    assert rel(oracle_mod.silu_mul(g, u), fix["silu_" + case[0]]) < 1e-6
