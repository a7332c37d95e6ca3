"""The Q4M layout and the tensor-core GEMV arithmetic, checked on the CPU: the numpy packer
is lossless, and the kernel's derivation (exact fp16 decode 1024 + s*q, x as fp16 hi + lo
with a power-of-two pre-scale, block-diagonal B, accumulator offset -(1024 + 8s) * sum(B))
reproduces the oracle's matvec (reference cuda/matmul_kernels.cu:8-43) within 1e-3."""
import ctypes as C

import numpy as np
import pytest

import q4m_ref
from oracle import oracle

REL = 1e-3


def q4_0_rows(rows, cols, seed, std=0.02):
    import jinf
    x = (np.random.default_rng(seed).standard_normal(rows * cols) * std).astype(np.float32)
    out = np.empty(rows * cols // 32 * 18, dtype=np.uint8)
    jinf.lib.jinf_quantize_q4_0(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), rows * cols)
    return out.reshape(rows, -1)


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def test_q4m_bytes_formula():
    import jinf
    for rows, cols in [(1, 128), (37, 384), (4096, 4096), (128256, 4096), (16, 96), (4096, 704)]:
        assert jinf.lib.jinf_b200_q4m_bytes(rows, cols) == ((rows + 31) // 32) * ((cols + 127) // 128) * 2304
    assert jinf.lib.jinf_b200_q4m_bytes(16, 100) == 0


def test_nibble_positions_are_a_permutation():
    bits = sorted(q4m_ref.nibble_bit(r, j) for r in (0, 8) for j in range(4))
    assert bits == list(range(0, 32, 4))


@pytest.mark.parametrize("rows,cols", [(16, 128), (37, 384), (100, 1408), (24, 704), (16, 96)])
def test_pack_is_lossless(rows, cols):
    w = q4_0_rows(rows, cols, seed=rows)
    img = q4m_ref.pack(w, rows, cols)
    tiles, groups = 2 * ((rows + 31) // 32), (cols + 127) // 128
    assert img.size == tiles * groups * 1152
    words, sc = q4m_ref.unpack_words(img, tiles, groups)
    # every nibble exactly once: rebuild the AoS qs bytes from the words
    blocks = w.reshape(rows, cols // 32, 18)
    got = np.zeros((tiles * 16, groups * 4, 32), dtype=np.uint8)
    for lane in range(32):
        gr, c = lane >> 2, lane & 3
        for i in range(8):
            for half in range(2):
                r = gr + 8 * half
                for j in range(4):
                    q = (words[:, :, lane, i] >> q4m_ref.nibble_bit(r, j)) & 15
                    rows_idx = np.arange(tiles) * 16 + r
                    got[rows_idx[:, None], np.arange(groups)[None, :] * 4 + j, 4 * i + c] = q
    want = np.empty((rows, cols // 32, 32), dtype=np.uint8)
    want[:, :, 0::2] = blocks[:, :, 2:] & 15
    want[:, :, 1::2] = blocks[:, :, 2:] >> 4
    assert np.array_equal(got[:rows, :cols // 32], want)
    assert not got[rows:].any() and not got[:, cols // 32:].any()


@pytest.mark.parametrize("rows,cols", [(16, 128), (37, 384), (64, 1024), (100, 1408), (48, 704), (16, 96)])
def test_emulated_gemv_matches_oracle(rows, cols):
    w = q4_0_rows(rows, cols, seed=rows + cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    y = q4m_ref.emulate_gemv(q4m_ref.pack(w, rows, cols), x, rows, cols)
    assert rel_err(y, oracle.matvec(w, 2, x, rows, cols)) < REL


def test_emulated_gemv_extreme_scales_and_inputs():
    rows, cols = 32, 512
    rng = np.random.default_rng(0)
    w = rng.integers(0, 256, size=(rows, cols // 32, 18), dtype=np.uint8)
    d = np.array([1e-7, 6e-5, 1.0, 300.0, -2.5, 65504.0], dtype=np.float16)
    w[..., 0:2] = np.frombuffer(rng.choice(d, size=rows * cols // 32).astype(np.float16).tobytes(),
                                dtype=np.uint8).reshape(rows, cols // 32, 2)
    w = w.reshape(rows, -1)
    for scale in (1e-6, 1.0, 1e5):
        x = (rng.standard_normal(cols) * scale).astype(np.float32)
        y = q4m_ref.emulate_gemv(q4m_ref.pack(w, rows, cols), x, rows, cols)
        assert rel_err(y, oracle.matvec(w, 2, x, rows, cols)) < REL
