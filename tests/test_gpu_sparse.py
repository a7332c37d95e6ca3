"""Sparse FFN modes of the engine on the GPU (reference
src/engine.cpp:339-415 forward_layer_sparse_ffn). The device predictor is checked against
numpy on the same fp16 weights (top-k ids identical away from exact score ties); decode
in both modes is checked against the CPU oracle whose FFN is restricted to the same
neurons (logits within 1e-2, greedy tokens identical)."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle
from test_gpu_engine import LOGIT_REL, rel_err
from test_sparse_host import fixed_mask

pytestmark = pytest.mark.gpu


def host_weights(seed, layer, which, n):
    import jinf
    out = np.empty(n, dtype=np.uint16)
    jinf.lib.jinf_sparse_predictor_weights(seed, layer, which, n, out.ctypes.data_as(C.c_void_p))
    return out.view(np.float16)


@pytest.mark.parametrize("d,r,ff,k", [(512, 128, 1408, 211), (4096, 1024, 14336, 2150)])
def test_predictor_topk_matches_numpy(cuda, d, r, ff, k):
    import jinf
    w1 = host_weights(5, 1, 1, r * d).reshape(r, d)
    w2 = host_weights(5, 1, 2, ff * r).reshape(ff, r)
    x = np.random.default_rng(d).standard_normal(d).astype(np.float32)
    bs = 1000
    ids = torch.empty(k, dtype=torch.int32, device=cuda)
    offs = torch.empty(k, dtype=torch.int32, device=cuda)
    scratch = torch.empty(r + ff, dtype=torch.float32, device=cuda)
    tw1, tw2, tx = (torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (w1, w2, x))
    st = jinf.lib.jinf_b200_sparse_predict(tw1.data_ptr(), tw2.data_ptr(), tx.data_ptr(), d, r, ff, k, bs,
                                           ids.data_ptr(), offs.data_ptr(), scratch.data_ptr(), None)
    assert st == 0
    torch.cuda.synchronize()
    z = np.maximum(w1.astype(np.float64) @ x.astype(np.float64), 0.0)
    s = w2.astype(np.float64) @ z
    got = ids.cpu().numpy()
    assert np.all(np.diff(got) > 0)
    assert np.array_equal(offs.cpu().numpy(), got * bs)
    # the device scores follow numpy to fp32 rounding; compare the sets away from the cut
    order = np.argsort(-s, kind="stable")
    thr = s[order[k - 1]]
    tol = 1e-4 * np.abs(s).max()
    sure_in = set(np.where(s > thr + tol)[0].tolist())
    sure_out = set(np.where(s < thr - tol)[0].tolist())
    g = set(got.tolist())
    assert sure_in <= g and not (g & sure_out)
    dev_s = scratch[r:].cpu().numpy()
    assert rel_err(dev_s, s) < 1e-4


@pytest.fixture(scope="module")
def tiny():
    import jinf
    return jinf.SynthModel(jinf.TINY, seed=0)


@pytest.fixture(scope="module")
def prompt():
    return [int(t) for t in np.random.default_rng(1).integers(0, 4096, size=12)]


@pytest.mark.parametrize("persistent", [True, False], ids=["persistent", "per_op"])
def test_sparse_fixed_mask_decode_matches_masked_oracle(cuda, tiny, prompt, persistent):
    """Fixed masks in both forms: the persistent step over gate|up and down compacted to the
    32-neuron blocks that hold an active neuron (inactive rows zeroed), and the kernel per
    operation over the reference's neuron bundles."""
    import jinf
    keep, seed = 0.15, 3
    eng = jinf.Engine.from_synth(tiny, max_context=96,
                                 options=jinf.b200_options(eos_token=-1, sparse_mode=2, sparse_keep=keep,
                                                           sparse_seed=seed, persistent=persistent))
    assert eng.persistent == persistent
    orc = oracle.OracleModel(tiny, max_ctx=96, kv_f16=True)
    for L in range(tiny.shape.n_layers):
        ids = fixed_mask(seed, L, tiny.shape.n_ff, keep)
        assert np.array_equal(eng.sparse_ids(L), ids)
        orc.set_ffn_mask(L, ids)
    want = None
    for t in prompt:
        want = orc.forward(t)
    got = eng.logits_host(prompt)
    assert rel_err(got, want) < LOGIT_REL
    for step in range(32):
        tok = oracle.argmax(want)
        assert eng.last_argmax() == tok, f"step {step}"
        want = orc.forward(tok)
        got = eng.logits_host([tok])
        assert rel_err(got, want) < LOGIT_REL, f"step {step}"


def test_sparse_predictor_decode_matches_oracle_on_its_neurons(cuda, tiny, prompt):
    import jinf
    eng = jinf.Engine.from_synth(tiny, max_context=96,
                                 options=jinf.b200_options(eos_token=-1, sparse_mode=1, sparse_keep=0.15))
    orc = oracle.OracleModel(tiny, max_ctx=96, kv_f16=True)
    k = int(np.floor(0.15 * tiny.shape.n_ff))
    toks = list(prompt)
    for step in range(len(prompt) + 16):
        t = toks[step]
        got = eng.logits_host([t])
        for L in range(tiny.shape.n_layers):
            ids = eng.sparse_ids(L)
            assert ids.size == k and np.all(np.diff(ids) > 0)
            orc.set_ffn_mask(L, ids)
        want = orc.forward(t)
        assert rel_err(got, want) < LOGIT_REL, f"step {step}"
        if step + 1 >= len(toks):
            toks.append(oracle.argmax(want))
            assert eng.last_argmax() == toks[-1], f"step {step}"


def test_sparse_modes_are_deterministic(cuda, tiny, prompt):
    import jinf
    outs = []
    for _ in range(2):
        eng = jinf.Engine.from_synth(tiny, max_context=96,
                                     options=jinf.b200_options(eos_token=-1, sparse_mode=1))
        outs.append(eng.generate(prompt, 24))
        eng.close()
    assert outs[0] == outs[1]


def test_sparse_mode_rejects_bad_options(cuda, tiny):
    import jinf
    for opts in (dict(sparse_mode=3), dict(sparse_mode=1, sparse_keep=0.0), dict(sparse_mode=2, sparse_keep=1.5)):
        with pytest.raises(jinf.JinfError):
            jinf.Engine.from_synth(tiny, max_context=32, options=jinf.b200_options(**opts))


def _cudart():
    for name in ("libcudart.so", "libcudart.so.12"):
        try:
            lib = C.CDLL(name)
            lib.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
            return lib
        except OSError:
            continue
    pytest.skip("no CUDA runtime library to copy the hook's gate")


def test_count_activations_matches_host_hook_counting(cuda, tiny, prompt):
    """Device-side calibration counts equal the reference tool's method: the FFN hook's gate
    copied to the host, |SiLU(g)| > threshold counted there (tools/profile_activations.cpp)."""
    import jinf
    from jinf import _lib as L
    thr = 0.05
    eng = jinf.Engine.from_synth(tiny, max_context=96, options=jinf.b200_options(eos_token=-1))
    n_layers, n_ff = tiny.shape.n_layers, tiny.shape.n_ff
    got = np.zeros((n_layers, n_ff), np.int32)
    eng.count_activations(prompt, thr, got)
    eng.reset()
    want = np.zeros((n_layers, n_ff), np.int64)
    rt = _cudart()
    buf = np.empty(n_ff, np.float32)

    def hook(_data, layer, gate, n):
        assert rt.cudaMemcpy(buf.ctypes.data, gate, 4 * n, 2) == 0
        g = buf[:n]
        silu = g / (np.float32(1.0) + np.exp(-g))
        want[layer, :n] += np.abs(silu) > np.float32(thr)

    cb = L.FFN_HOOK(hook)
    eng.h.contents.ffn_hook = cb
    eng.logits_host(prompt)
    eng.h.contents.ffn_hook = L.FFN_HOOK()
    eng.close()
    assert got.sum() > 0
    # expf on the device and exp on the host may round a value at the threshold differently
    assert np.sum(got != want) <= 2, np.argwhere(got != want)[:8]


def test_predictor_path_static_profile_matches_oracle(cuda, tiny, prompt, tmp_path):
    """jinf_engine_config.predictor_path: the reference's static predictor (neurons whose
    profiled frequency exceeds sparsity_threshold), in the persistent step."""
    import jinf
    from jinf.calibrate import write_profile
    n_layers, n_ff = tiny.shape.n_layers, tiny.shape.n_ff
    rng = np.random.default_rng(9)
    counts = rng.integers(0, 1000, size=(n_layers, n_ff)).astype(np.int32)
    path = str(tmp_path / "act.bin")
    write_profile(path, counts, 1000)
    thr = 0.8
    eng = jinf.Engine.from_synth(tiny, max_context=96, options=jinf.b200_options(eos_token=-1),
                                 predictor_path=path, sparsity_threshold=thr)
    assert eng.persistent
    orc = oracle.OracleModel(tiny, max_ctx=96, kv_f16=True)
    for L in range(n_layers):
        ids = np.nonzero(counts[L].astype(np.float32) / np.float32(1000) > np.float32(thr))[0]
        assert np.array_equal(eng.sparse_ids(L), ids)
        orc.set_ffn_mask(L, ids.astype(np.int32))
    want = None
    for t in prompt:
        want = orc.forward(t)
    got = eng.logits_host(prompt)
    assert rel_err(got, want) < LOGIT_REL
    for step in range(8):
        tok = oracle.argmax(want)
        assert eng.last_argmax() == tok, f"step {step}"
        want = orc.forward(tok)
        got = eng.logits_host([tok])
        assert rel_err(got, want) < LOGIT_REL, f"step {step}"


def test_predictor_path_that_cannot_be_read_leaves_the_ffn_dense(cuda, tiny, prompt, tmp_path):
    import jinf
    eng = jinf.Engine.from_synth(tiny, max_context=96, options=jinf.b200_options(eos_token=-1),
                                 predictor_path=str(tmp_path / "missing.bin"))
    with pytest.raises(Exception):
        eng.sparse_ids(0)
    orc = oracle.OracleModel(tiny, max_ctx=96, kv_f16=True)
    want = None
    for t in prompt:
        want = orc.forward(t)
    assert rel_err(eng.logits_host(prompt), want) < LOGIT_REL
