"""Parity at the positions and sizes the benchmark quotes (C3: Llama-3-8B shape, Q4_0,
positions 512 and beyond), against the CPU oracle.

At position ~520 the persistent step's attention cuts each of the 8 kv heads into 18 splits
and merges them cooperatively; these tests run that regime. Both sides start from the same
512-position KV cache: the engine fills it with seeded values, the oracle loads the engine's
cache bytes (Engine.kv_read / OracleModel.load_kv_f16), and from there both compute every
token themselves (KV rows of the new positions included).

Bars: logits within 1e-2 max relative error, greedy tokens identical;
the smallest top-1/top-2 logit gap of the oracle is printed.
"""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

LOGIT_REL = 1e-2
KV_POS = 512


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def top_gap(v):
    t = np.sort(v)[-2:]
    return float(t[1] - t[0])


def run_from_cache(eng, orc, prompt, n_steps, kv_pos=KV_POS):
    """The engine's cache -> the oracle, then the prompt, then n_steps greedy tokens on both;
    returns (max relative logits error, min top-1/top-2 gap)."""
    k, v = eng.kv_read(kv_pos)
    orc.load_kv_f16(k, v)
    want = None
    for t in prompt:
        want = orc.forward(t)
    got = eng.logits_host(prompt)
    assert eng.n_past == kv_pos + len(prompt)
    worst, gap = rel_err(got, want), top_gap(want)
    assert worst < LOGIT_REL
    for step in range(n_steps):
        tok = oracle.argmax(want)
        assert eng.last_argmax() == tok, f"step {step}: engine {eng.last_argmax()} oracle {tok} (gap {top_gap(want):.3g})"
        want = orc.forward(tok)
        got = eng.logits_host([tok])
        e = rel_err(got, want)
        assert e < LOGIT_REL, f"step {step}: logits relative error {e:.3g}"
        worst, gap = max(worst, e), min(gap, top_gap(want))
    return worst, gap


@pytest.mark.parametrize("persistent", [pytest.param(True, id="persistent"), pytest.param(False, id="per_op")])
def test_8b_shaped_layers_at_bench_positions_32_greedy(cuda, persistent):
    """Two 8B-shaped layers (d 4096, 32/8 heads of 128, ff 14336, theta 5e5; vocabulary
    32000) at positions 512..547: 4 prompt tokens, then 32 greedy steps."""
    import jinf
    shape = jinf.LlamaShape(2, 4096, 32, 8, 14336, 32000, 5e5)
    syn = jinf.SynthModel(shape, seed=5)
    eng = jinf.Engine.from_synth(syn, max_context=KV_POS + 48,
                                 options=jinf.b200_options(eos_token=-1, persistent=persistent))
    assert eng.persistent == persistent
    eng.fill_kv_random(KV_POS, seed=1)
    orc = oracle.OracleModel(syn, max_ctx=KV_POS + 48, kv_f16=True)
    prompt = [int(t) for t in np.random.default_rng(2).integers(0, shape.n_vocab, size=4)]
    worst, gap = run_from_cache(eng, orc, prompt, 32)
    print(f"8B-shaped x2 layers, positions {KV_POS}..{KV_POS + 35}: max logits rel err {worst:.3g}, "
          f"min top-1/top-2 gap {gap:.3g}")
    orc.close()
    eng.close()


def test_full_c3_model_at_bench_positions(cuda):
    """The whole C3 model the benchmark times (32 layers, vocabulary 128256, the bench's
    seed-0 weights) in the persistent step, positions 512..523: 4 prompt tokens and 8
    greedy steps. Covers the LM-head partition over 128256 rows inside the step kernel."""
    import jinf
    syn = jinf.SynthModel(jinf.LLAMA3_8B, seed=0)
    eng = jinf.Engine.from_synth(syn, max_context=KV_POS + 16, options=jinf.b200_options(eos_token=-1))
    assert eng.persistent
    eng.fill_kv_random(KV_POS, seed=1)
    orc = oracle.OracleModel(syn, max_ctx=KV_POS + 16, kv_f16=True)
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, jinf.LLAMA3_8B.n_vocab, size=4)]
    worst, gap = run_from_cache(eng, orc, prompt, 8)
    print(f"C3 8B model, positions {KV_POS}..{KV_POS + 11}: max logits rel err {worst:.3g}, "
          f"min top-1/top-2 gap {gap:.3g}")
    orc.close()
    eng.close()


def test_70b_shaped_layers_at_8192_positions(cuda):
    """Two layers of the 70B shape (d 8192, 64/8 heads of 128, ff 28672, Q4_K weights;
    vocabulary 32000) over a KV cache filled to 8192 positions (config C5's context): the
    attention splits every kv head 18 ways over 513-position splits. 4 prompt tokens, then 8
    greedy steps."""
    import jinf
    from jinf import _lib as L
    shape = jinf.LlamaShape(2, 8192, 64, 8, 28672, 32000, 5e5)
    syn = jinf.SynthModel(shape, seed=7, weight_type=L.Q4_K)
    eng = jinf.Engine.from_synth(syn, max_context=8192 + 16, options=jinf.b200_options(eos_token=-1))
    assert eng.persistent
    eng.fill_kv_random(8192, seed=1)
    orc = oracle.OracleModel(syn, max_ctx=8192 + 16, kv_f16=True)
    prompt = [int(t) for t in np.random.default_rng(3).integers(0, shape.n_vocab, size=4)]
    worst, gap = run_from_cache(eng, orc, prompt, 8, kv_pos=8192)
    print(f"70B-shaped x2 layers, positions 8192..8203: max logits rel err {worst:.3g}, min top-1/top-2 gap {gap:.3g}")
    orc.close()
    eng.close()
