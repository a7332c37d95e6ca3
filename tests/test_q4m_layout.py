"""The Q4M layout and the tensor-core GEMV arithmetic, checked on the CPU: the numpy packer
is lossless, and the kernel's derivation (u8 weights, x as two int8 digits per element with
a per-block scale, exact integer block sums with the zero point removed through the
accumulator's start value) reproduces the oracle's matvec (reference
cuda/matmul_kernels.cu:8-43) within 1e-3."""
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
    off = q4m_ref._layout()[:16].reshape(-1)   # tile A rows; tile B shares the bytes (high nibbles)
    assert np.array_equal(np.sort(off), np.arange(2048))


@pytest.mark.parametrize("rows,cols", [(16, 128), (37, 384), (100, 1408), (24, 704), (16, 96), (64, 256)])
def test_pack_is_lossless(rows, cols):
    w = q4_0_rows(rows, cols, seed=rows)
    img = q4m_ref.pack(w, rows, cols)
    pairs, groups = (rows + 31) // 32, (cols + 127) // 128
    assert img.size == pairs * groups * 2304
    q, d = q4m_ref.unpack(img, rows, cols)
    blocks = w.reshape(rows, cols // 32, 18)
    want = np.empty((rows, cols // 32, 32), dtype=np.uint8)
    want[:, :, 0::2] = blocks[:, :, 2:] & 15
    want[:, :, 1::2] = blocks[:, :, 2:] >> 4
    assert np.array_equal(q[:, :cols // 32], want)
    assert np.array_equal(d[:, :cols // 32], blocks[:, :, 0].astype(np.uint16) | (blocks[:, :, 1].astype(np.uint16) << 8))
    assert not q[:, cols // 32:].any() and not d[:, cols // 32:].any()
    # rows past `rows` are zero in the image: repacking with them dropped changes nothing
    full = q4m_ref.pack(np.concatenate([w, np.zeros((pairs * 32 - rows, w.shape[1]), np.uint8)]), pairs * 32, cols)
    assert np.array_equal(full, img)


def test_digit_records_round_trip():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(384) * np.repeat(10.0 ** rng.integers(-6, 6, size=12), 32)).astype(np.float32)
    x[64:96] = 0.0                              # an all-zero block
    hi, lo, inv_alpha = q4m_ref.x_records(x, 384)
    back = ((256 * hi + lo) * inv_alpha[:, None]).reshape(-1)
    amax = np.repeat(np.max(np.abs(x.reshape(-1, 32)), axis=1), 32)
    assert np.all(np.abs(back - x) <= amax * 2.0 ** -15)


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
        x[128:160] = 0.0
        y = q4m_ref.emulate_gemv(q4m_ref.pack(w, rows, cols), x, rows, cols)
        assert rel_err(y, oracle.matvec(w, 2, x, rows, cols)) < REL


def q4_k_rows(rows, cols, seed, std=0.02):
    import jinf
    x = (np.random.default_rng(seed).standard_normal(rows * cols) * std).astype(np.float32)
    out = np.empty(rows * cols // 256 * 144, dtype=np.uint8)
    jinf.lib.jinf_quantize_q4_K(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), rows * cols)
    return out.reshape(rows, -1)


@pytest.mark.parametrize("rows,cols", [(16, 256), (37, 512), (100, 1024), (64, 768)])
def test_pack_q4k_is_lossless(rows, cols):
    w = q4_k_rows(rows, cols, seed=rows)
    img = q4m_ref.pack_q4k(w, rows, cols)
    assert img.size == ((rows + 31) // 32) * (cols // 128) * 2432
    q, sc, mn, d, dmin = q4m_ref.unpack_q4k(img, rows, cols)
    wq, wsc, wmn, wd, wdmin = q4m_ref._q4k_fields(w, rows, cols)
    assert np.array_equal(q, wq) and np.array_equal(sc, wsc) and np.array_equal(mn, wmn)
    assert np.array_equal(d, np.repeat(wd, 8, axis=1)) and np.array_equal(dmin, np.repeat(wdmin, 8, axis=1))


@pytest.mark.parametrize("rows,cols", [(16, 256), (37, 512), (64, 1024), (100, 2048)])
def test_emulated_gemv_q4k_matches_oracle(rows, cols):
    w = q4_k_rows(rows, cols, seed=rows + cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    y = q4m_ref.emulate_gemv_q4k(q4m_ref.pack_q4k(w, rows, cols), x, rows, cols)
    assert rel_err(y, oracle.matvec(w, 12, x, rows, cols)) < REL


# ---------------------------------------------------------------- Q6_K and Q8_0 units

@pytest.mark.parametrize("rows,cols", [(16, 256), (37, 512), (64, 1024), (100, 768)])
def test_emulated_gemv_q6k_matches_oracle(rows, cols):
    w = q4m_ref.random_q6k_rows(rows, cols, seed=rows + cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    img = q4m_ref.pack_q6k(w, rows, cols)
    assert img.size == ((rows + 31) // 32) * (cols // 128) * 3392
    y = q4m_ref.emulate_gemv_q6k(img, x, rows, cols)
    assert rel_err(y, oracle.matvec(w, 14, x, rows, cols)) < REL


@pytest.mark.parametrize("rows,cols", [(16, 32), (37, 160), (64, 1024), (100, 736)])
def test_emulated_gemv_q80_matches_oracle(rows, cols):
    w = q4m_ref.random_q80_rows(rows, cols, seed=rows + cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    img = q4m_ref.pack_q80(w, rows, cols)
    assert img.size == ((rows + 31) // 32) * ((cols + 127) // 128) * 4352
    y = q4m_ref.emulate_gemv_q80(img, x, rows, cols)
    assert rel_err(y, oracle.matvec(w, 8, x, rows, cols)) < REL


@pytest.mark.parametrize("qt,fn,bb,bs", [(8, "jinf_quantize_q8_0", 34, 32), (14, "jinf_quantize_q6_K", 210, 256)])
def test_host_quantizers_round_trip(qt, fn, bb, bs):
    """The synthetic-model quantizers for Q8_0 and Q6_K: dequantized (oracle) values lie within
    half a quantisation step (plus fp16 rounding of the scales) of the input."""
    import jinf
    n = 4096
    x = (np.random.default_rng(qt).standard_normal(n) * 0.02).astype(np.float32)
    out = np.zeros(n // bs * bb, dtype=np.uint8)
    getattr(jinf.lib, fn)(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), n)
    y = oracle.dequant(out, qt)
    err = np.abs(y - x).reshape(-1, 16 if qt == 14 else 32).max(axis=1)
    amax = np.abs(x).reshape(-1, 16 if qt == 14 else 32).max(axis=1)
    steps = 31.0 if qt == 14 else 127.0
    assert np.all(err <= amax / steps * 0.55 + 1e-6), float(np.max(err / (amax / steps)))


def test_synth_mixed_types():
    """mix_type puts attn_v and ffn_down of the even layers and the output head in the second
    type, the Q4_K_M pattern; everything else keeps weight_type."""
    import jinf
    from jinf import _lib as L
    syn = jinf.SynthModel(jinf.LlamaShape(4, 512, 8, 2, 1536, 4096, 10000.0, 1e-5), seed=0,
                          weight_type=L.Q4_K, mix_type=L.Q6_K)
    for name in syn.tensor_names():
        t = syn.tensor_info(name)[0]
        if name.endswith("norm.weight") or name == "token_embd.weight":
            assert t == L.F32
        elif name == "output.weight" or (name.split(".")[-2] in ("attn_v", "ffn_down") and int(name.split(".")[1]) % 2 == 0):
            assert t == L.Q6_K, name
        else:
            assert t == L.Q4_K, name


@pytest.mark.parametrize("qt,rows,cols", [(2, 37, 384), (2, 100, 1408), (12, 37, 512), (14, 100, 768), (8, 40, 96),
                                          (8, 64, 1024)])
def test_host_pack_matches_layout(qt, rows, cols):
    """jinf_b200_q4m_pack_host (the device repack's lane functions run on the host) writes the
    documented layout, byte for byte."""
    import jinf
    if qt == 2:
        w, ref = q4_0_rows(rows, cols, seed=rows), q4m_ref.pack
    elif qt == 12:
        w, ref = q4_k_rows(rows, cols, seed=rows), q4m_ref.pack_q4k
    elif qt == 14:
        w, ref = q4m_ref.random_q6k_rows(rows, cols, seed=rows), q4m_ref.pack_q6k
    else:
        w, ref = q4m_ref.random_q80_rows(rows, cols, seed=rows), q4m_ref.pack_q80
    w = np.ascontiguousarray(w)
    out = np.full(jinf.lib.jinf_b200_q4m_bytes_qt(rows, cols, qt), 0xAB, dtype=np.uint8)
    assert jinf.lib.jinf_b200_q4m_pack_host(w.ctypes.data_as(C.c_void_p), qt, out.ctypes.data_as(C.c_void_p),
                                            rows, cols) == 0
    assert np.array_equal(out, ref(w, rows, cols))


def step_unit_offset(u, split_pairs, groups, unit_a, unit_b):
    """Byte offset of unit u (pair-major: pair u // groups, group u % groups) in a persistent-step
    phase whose first `split_pairs` pairs are in a format with unit_a-byte units and the rest
    in one with unit_b-byte units (the step kernel's stream position and its L2 prefetch of a
    CTA's unit range, csrc/step_kernel.cu)."""
    cs = split_pairs * groups
    return u * unit_a if u <= cs else cs * unit_a + (u - cs) * unit_b


def test_split_phase_unit_offsets_match_the_packed_images():
    """A QKV phase of a Q4_K_M-like layer streams [q | k] in Q4_K then v in Q6_K from one buffer:
    the two host-packed images side by side. Every unit the offset rule addresses is that
    image's unit (pair, group), at the packer's own offset ((pair * groups + group) * unit)."""
    import jinf
    rows_qk, rows_v, cols = 96, 32, 512
    groups = cols // 128
    wa = np.ascontiguousarray(q4_k_rows(rows_qk, cols, seed=1))
    wb = np.ascontiguousarray(q4m_ref.random_q6k_rows(rows_v, cols, seed=2))
    ia = np.zeros(jinf.lib.jinf_b200_q4m_bytes_qt(rows_qk, cols, 12), dtype=np.uint8)
    ib = np.zeros(jinf.lib.jinf_b200_q4m_bytes_qt(rows_v, cols, 14), dtype=np.uint8)
    assert jinf.lib.jinf_b200_q4m_pack_host(wa.ctypes.data_as(C.c_void_p), 12, ia.ctypes.data_as(C.c_void_p),
                                            rows_qk, cols) == 0
    assert jinf.lib.jinf_b200_q4m_pack_host(wb.ctypes.data_as(C.c_void_p), 14, ib.ctypes.data_as(C.c_void_p),
                                            rows_v, cols) == 0
    ua, ub = ia.size // (rows_qk // 32 * groups), ib.size // (rows_v // 32 * groups)
    assert (ua, ub) == (2432, 3392)
    buf = np.concatenate([ia, ib])
    pa = rows_qk // 32
    for u in range((pa + rows_v // 32) * groups):
        o = step_unit_offset(u, pa, groups, ua, ub)
        p, g = divmod(u, groups)
        want = ia[(p * groups + g) * ua:][:ua] if p < pa else ib[((p - pa) * groups + g) * ub:][:ub]
        assert np.array_equal(buf[o:o + want.size], want), u
    assert step_unit_offset((pa + rows_v // 32) * groups, pa, groups, ua, ub) == buf.size
