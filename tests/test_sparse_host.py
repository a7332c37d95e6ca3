"""Host side of the engine's sparse-FFN modes (reference src/engine.cpp:339-415,
src/activation_predictor.cpp): the fixed neuron masks (runs of 8 kept with probability
`keep`, BASELINE config C4's fixed-mask variant), the seeded predictor weights, and the
oracle's masked FFN (non-selected neurons contribute nothing)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle


def fixed_mask(seed, layer, n_ff, keep):
    import jinf
    n = jinf.lib.jinf_sparse_fixed_mask(seed, layer, n_ff, keep, None)
    ids = np.empty(n, dtype=np.int32)
    assert jinf.lib.jinf_sparse_fixed_mask(seed, layer, n_ff, keep, ids.ctypes.data_as(C.c_void_p)) == n
    return ids


def test_fixed_mask_is_runs_of_8_sorted_and_about_keep():
    ids = fixed_mask(0, 3, 14336, 0.15)
    assert np.all(np.diff(ids) > 0)
    runs = np.unique(ids // 8)
    assert np.array_equal(np.sort(ids), np.sort((runs[:, None] * 8 + np.arange(8)).reshape(-1)))
    frac = ids.size / 14336
    assert abs(frac - 0.15) < 0.03
    assert np.array_equal(ids, fixed_mask(0, 3, 14336, 0.15))        # deterministic
    assert not np.array_equal(ids, fixed_mask(0, 4, 14336, 0.15))    # per layer
    assert not np.array_equal(ids, fixed_mask(1, 3, 14336, 0.15))    # per seed
    assert fixed_mask(0, 0, 1408, 1.0).size == 1408 and fixed_mask(0, 0, 100, 1.0).size == 100


def test_predictor_weights_are_seeded_normals():
    import jinf
    n = 1 << 16
    a = np.empty(n, dtype=np.uint16)
    b = np.empty(n, dtype=np.uint16)
    jinf.lib.jinf_sparse_predictor_weights(7, 2, 1, n, a.ctypes.data_as(C.c_void_p))
    jinf.lib.jinf_sparse_predictor_weights(7, 2, 1, n, b.ctypes.data_as(C.c_void_p))
    assert np.array_equal(a, b)
    v = a.view(np.float16).astype(np.float64)
    assert abs(v.std() - 0.02) < 0.001 and abs(v.mean()) < 0.001
    jinf.lib.jinf_sparse_predictor_weights(7, 2, 2, n, b.ctypes.data_as(C.c_void_p))
    assert not np.array_equal(a, b)


def test_oracle_mask_of_every_neuron_is_the_dense_ffn():
    import jinf
    syn = jinf.SynthModel(jinf.LlamaShape(2, 256, 4, 2, 512, 1024, 10000.0, 1e-5), seed=0)
    dense = oracle.OracleModel(syn, max_ctx=8)
    masked = oracle.OracleModel(syn, max_ctx=8)
    none = oracle.OracleModel(syn, max_ctx=8)
    for L in range(2):
        masked.set_ffn_mask(L, np.arange(512))
        none.set_ffn_mask(L, np.array([], dtype=np.int32))
    for t in (3, 5):
        a, b, c = dense.forward(t), masked.forward(t), none.forward(t)
    assert np.array_equal(a, b)
    assert not np.allclose(a, c)
