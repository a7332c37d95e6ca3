"""Multi-sequence decode (jinf_engine_decode_batch): up to 8 sequences, each with its own KV
cache and position, advanced by one token per step with every projection's weights streamed
once for all of them. Each sequence is checked against its own CPU oracle model decoding it
alone (the reference's one-sequence loop, src/engine.cpp:691-751).

Bars: logits within 1e-2 max relative error, greedy tokens identical; the smallest
top-1/top-2 logit gap of the oracle is printed."""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

LOGIT_REL = 1e-2


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def top_gap(v):
    t = np.sort(v)[-2:]
    return float(t[1] - t[0])


def run_lockstep(eng, orcs, seqs, prompts, n_greedy):
    """Feed every sequence's prompt one token per step (all sequences in each step), then
    n_greedy greedy steps; every step's logits and argmax against each sequence's oracle.
    Returns (max relative logits error, min top-1/top-2 gap)."""
    worst, gap = 0.0, float("inf")
    want = [None] * len(seqs)
    for t in range(len(prompts[0])):
        toks = [p[t] for p in prompts]
        got_tok, got = eng.decode_batch(seqs, toks, want_logits=True)
        for i, orc in enumerate(orcs):
            want[i] = orc.forward(toks[i])
            e = rel_err(got[i], want[i])
            assert e < LOGIT_REL, f"prompt {t} sequence {seqs[i]}: {e:.3g}"
            assert got_tok[i] == oracle.argmax(want[i]), f"prompt {t} sequence {seqs[i]}"
            worst, gap = max(worst, e), min(gap, top_gap(want[i]))
    for step in range(n_greedy):
        toks = [oracle.argmax(w) for w in want]
        got_tok, got = eng.decode_batch(seqs, toks, want_logits=True)
        for i, orc in enumerate(orcs):
            want[i] = orc.forward(toks[i])
            e = rel_err(got[i], want[i])
            assert e < LOGIT_REL, f"step {step} sequence {seqs[i]}: {e:.3g}"
            assert got_tok[i] == oracle.argmax(want[i]), f"step {step} sequence {seqs[i]} (gap {top_gap(want[i]):.3g})"
            worst, gap = max(worst, e), min(gap, top_gap(want[i]))
    return worst, gap


def test_tiny_three_sequences_32_greedy(cuda):
    """C1 tiny model, three sequences with different 16-token prompts decoded together, then
    32 greedy steps; each matches its own oracle decode."""
    import jinf
    syn = jinf.SynthModel(jinf.TINY, seed=0)
    eng = jinf.Engine.from_synth(syn, max_context=128, options=jinf.b200_options(eos_token=-1, max_seqs=4))
    rng = np.random.default_rng(0)
    seqs = [0, 2, 3]
    prompts = [[int(t) for t in rng.integers(0, 4096, size=16)] for _ in seqs]
    orcs = [oracle.OracleModel(syn, max_ctx=128, kv_f16=True) for _ in seqs]
    worst, gap = run_lockstep(eng, orcs, seqs, prompts, 32)
    assert [eng.seq_n_past(s) for s in seqs] == [48, 48, 48]
    assert eng.seq_n_past(1) == 0 and eng.n_past == 48
    print(f"tiny x3 sequences: max logits rel err {worst:.3g}, min top-1/top-2 gap {gap:.3g}")
    for o in orcs:
        o.close()
    eng.close()


@pytest.mark.parametrize("qtype", ["q4_0", "q4_k"])
def test_8b_layers_eight_sequences_at_512(cuda, qtype):
    """Two 8B-shaped layers (d 4096, 32/8 heads, ff 14336; vocabulary 32000), eight sequences,
    each cache filled to 512 positions with its own seeded values (the oracles load the
    engine's bytes), then 2 prompt tokens and 6 greedy steps for all eight at once."""
    import jinf
    from jinf import _lib as L
    shape = jinf.LlamaShape(2, 4096, 32, 8, 14336, 32000, 5e5)
    syn = jinf.SynthModel(shape, seed=11, weight_type=L.Q4_0 if qtype == "q4_0" else L.Q4_K)
    ctx = 512 + 16
    eng = jinf.Engine.from_synth(syn, max_context=ctx, options=jinf.b200_options(eos_token=-1, max_seqs=8))
    seqs = list(range(8))
    orcs = []
    for s in seqs:
        eng.seq_fill_kv_random(s, 512, seed=100 + s)
        o = oracle.OracleModel(syn, max_ctx=ctx, kv_f16=True)
        o.load_kv_f16(*eng.seq_kv_read(s, 512))
        orcs.append(o)
    rng = np.random.default_rng(4)
    prompts = [[int(t) for t in rng.integers(0, shape.n_vocab, size=2)] for _ in seqs]
    worst, gap = run_lockstep(eng, orcs, seqs, prompts, 6)
    print(f"8B-shaped x2 layers ({qtype}), 8 sequences at 512..519: max logits rel err {worst:.3g}, "
          f"min top-1/top-2 gap {gap:.3g}")
    for o in orcs:
        o.close()
    eng.close()


@pytest.mark.parametrize("head_dim", [64, 128])
def test_eight_query_heads_per_kv_head_ragged_caches(cuda, head_dim):
    """Eight query heads per kv head (the 70B grouping) at head dims 64 and 128, four sequences
    whose caches hold 63, 64, 700 and 1500 seeded positions (one short of a 64-position block,
    exactly one block, and many blocks over several splits), then 1 prompt token and 3 greedy
    steps each, against each sequence's oracle."""
    import jinf
    shape = jinf.LlamaShape(2, 16 * head_dim, 16, 2, 2816, 4096, 5e5)
    syn = jinf.SynthModel(shape, seed=21 + head_dim)
    fills = [63, 64, 700, 1500]
    ctx = max(fills) + 8
    eng = jinf.Engine.from_synth(syn, max_context=ctx, options=jinf.b200_options(eos_token=-1, max_seqs=4))
    seqs = [0, 1, 2, 3]
    orcs = []
    for s, f in zip(seqs, fills):
        eng.seq_fill_kv_random(s, f, seed=300 + s)
        o = oracle.OracleModel(syn, max_ctx=ctx, kv_f16=True)
        o.load_kv_f16(*eng.seq_kv_read(s, f))
        orcs.append(o)
    rng = np.random.default_rng(head_dim)
    prompts = [[int(rng.integers(0, shape.n_vocab))] for _ in seqs]
    worst, gap = run_lockstep(eng, orcs, seqs, prompts, 3)
    print(f"GQA 8, head dim {head_dim}, caches {fills}: max logits rel err {worst:.3g}, min top-1/top-2 gap {gap:.3g}")
    for o in orcs:
        o.close()
    eng.close()


def test_ragged_positions_and_counts(cuda):
    """Sequences at different positions, stepped in changing subsets (1, 2, 3 and 5 vectors:
    one captured graph per count), each against its own oracle."""
    import jinf
    shape = jinf.LlamaShape(2, 512, 8, 2, 1408, 4096, 1e4)
    syn = jinf.SynthModel(shape, seed=3)
    eng = jinf.Engine.from_synth(syn, max_context=96, options=jinf.b200_options(eos_token=-1, max_seqs=5))
    orcs = [oracle.OracleModel(syn, max_ctx=96, kv_f16=True) for _ in range(5)]
    rng = np.random.default_rng(9)
    last = [None] * 5
    schedule = [[0], [1, 0], [2, 4, 1], [3], [0, 1, 2, 3, 4], [4, 2], [1, 3, 0, 2, 4], [2]]
    worst = 0.0
    for rnd in range(3):
        for group in schedule:
            toks = [int(rng.integers(0, shape.n_vocab)) if last[s] is None or rnd == 0 else oracle.argmax(last[s])
                    for s in group]
            got_tok, got = eng.decode_batch(group, toks, want_logits=True)
            for i, s in enumerate(group):
                last[s] = orcs[s].forward(toks[i])
                e = rel_err(got[i], last[s])
                assert e < LOGIT_REL, f"round {rnd} group {group} sequence {s}: {e:.3g}"
                assert got_tok[i] == oracle.argmax(last[s])
                worst = max(worst, e)
    for s in range(5):
        assert eng.seq_n_past(s) == orcs[s].pos
    print(f"ragged sequences: max logits rel err {worst:.3g}")
    for o in orcs:
        o.close()
    eng.close()


@pytest.mark.parametrize("persistent", [True, False])
def test_sequence_zero_shares_the_one_sequence_state(cuda, persistent):
    """Sequence 0 is the one forward() decodes: a prompt fed through decode_batch and then
    continued with forward() (and the reverse) gives the oracle's logits throughout."""
    import jinf
    syn = jinf.SynthModel(jinf.TINY, seed=1)
    eng = jinf.Engine.from_synth(syn, max_context=64,
                                 options=jinf.b200_options(eos_token=-1, max_seqs=2, persistent=persistent))
    orc = oracle.OracleModel(syn, max_ctx=64, kv_f16=True)
    rng = np.random.default_rng(2)
    toks = [int(t) for t in rng.integers(0, 4096, size=12)]
    for i, t in enumerate(toks):
        want = orc.forward(t)
        if i % 4 < 2:
            _, got = eng.decode_batch([0], [t], want_logits=True)
            got = got[0]
        else:
            got = eng.logits_host([t])
        assert rel_err(got, want) < LOGIT_REL, f"token {i}"
    assert eng.n_past == 12 and eng.seq_n_past(0) == 12
    orc.close()
    eng.close()


def test_decode_batch_rejects_bad_arguments(cuda):
    import jinf
    from jinf import _lib as L
    syn = jinf.SynthModel(jinf.TINY, seed=0)
    eng = jinf.Engine.from_synth(syn, max_context=8, options=jinf.b200_options(eos_token=-1, max_seqs=2))
    for seqs, toks in (([0, 0], [1, 2]), ([2], [1]), ([0], [4096]), ([-1], [1]), ([0, 1, 0], [1, 1, 1])):
        with pytest.raises(L.JinfError):
            eng.decode_batch(seqs, toks)
    for _ in range(8):
        eng.decode_batch([1], [5])
    with pytest.raises(L.JinfError):  # sequence 1's context is full
        eng.decode_batch([1], [5])
    eng.seq_reset(1)
    assert eng.seq_n_past(1) == 0
    eng.decode_batch([1], [5])
    eng.close()


def test_resident_matches_host_fed_steps(cuda):
    """decode_batch_resident (argmax fed back on the device) gives the tokens that host-fed
    decode_batch steps give, and leaves the same positions."""
    import jinf
    shape = jinf.LlamaShape(2, 512, 8, 2, 1408, 4096, 1e4)
    syn = jinf.SynthModel(shape, seed=5)
    seqs = [3, 0, 1]
    a = jinf.Engine.from_synth(syn, max_context=64, options=jinf.b200_options(eos_token=-1, max_seqs=4))
    b = jinf.Engine.from_synth(syn, max_context=64, options=jinf.b200_options(eos_token=-1, max_seqs=4))
    for eng in (a, b):
        for s in seqs:
            eng.seq_fill_kv_random(s, 10 + s, seed=s)
    first = [7, 99, 2048]
    got = a.decode_batch_resident(seqs, first, 20, collect=True)
    toks, want = first, []
    for _ in range(20):
        toks = b.decode_batch(seqs, toks)
        want.append(toks)
    assert got == want
    assert [a.seq_n_past(s) for s in seqs] == [b.seq_n_past(s) for s in seqs] == [10 + s + 20 for s in seqs]
    a.close()
    b.close()
