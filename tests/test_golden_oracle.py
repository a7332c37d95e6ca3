"""Pin the CPU oracle (and the library's host dequantizers) to golden vectors produced
by the reference's own src/quant.cpp (tests/golden/make_golden.py)."""
import ctypes as C
import hashlib

import numpy as np
import pytest

from oracle import oracle

KINDS = [("q4_0", 2, 32), ("q8_0", 8, 32), ("q4_K", 12, 256)]


@pytest.mark.parametrize("kind,qt,per", KINDS)
def test_oracle_dequant_bit_exact(golden, kind, qt, per):
    b = golden[f"{kind}_blocks"]
    ref = golden[f"{kind}_out"]
    got = oracle.dequant(b, qt)
    assert got.shape == ref.shape
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), "oracle dequant differs from the reference bits"


@pytest.mark.parametrize("kind,qt,per", KINDS)
def test_library_host_dequant_bit_exact(golden, kind, qt, per):
    import jinf
    b = np.ascontiguousarray(golden[f"{kind}_blocks"])
    ref = golden[f"{kind}_out"]
    out = np.empty_like(ref)
    fn = {"q4_0": jinf.lib.jinf_dequantize_q4_0, "q8_0": jinf.lib.jinf_dequantize_q8_0,
          "q4_K": jinf.lib.jinf_dequantize_q4_K}[kind]
    fn(b.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), b.shape[0])
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_fp16_all_values(golden):
    import jinf
    h = np.arange(65536, dtype=np.uint16)
    out = np.empty(65536, dtype=np.float32)
    jinf.lib.jinf_dequantize(h.ctypes.data_as(C.c_void_p), jinf.F16, out.ctypes.data_as(C.c_void_p), 65536)
    assert hashlib.sha256(out.tobytes()).digest() == bytes(golden["f16_all_sha256"])
    orc = oracle.fp16_to_fp32(np.arange(65536, dtype=np.uint16))
    assert hashlib.sha256(orc.tobytes()).digest() == bytes(golden["f16_all_sha256"])


def test_dispatcher_unknown_type_leaves_output():
    import jinf
    src = np.zeros(64, dtype=np.uint8)
    out = np.full(32, 7.0, dtype=np.float32)
    jinf.lib.jinf_dequantize(src.ctypes.data_as(C.c_void_p), 3, out.ctypes.data_as(C.c_void_p), 32)  # Q4_1
    assert np.all(out == 7.0)


def test_against_live_reference_random_blocks():
    """Extra seeds checked directly against the compiled reference, when it is present."""
    ref = oracle.ref_lib()
    if ref is None:
        pytest.skip("reference library not built here")
    rng = np.random.default_rng(1234)
    for qt, bb, per, fn in [(2, 18, 32, ref.ref_dequantize_q4_0), (12, 144, 256, ref.ref_dequantize_q4_K),
                            (8, 34, 32, ref.ref_dequantize_q8_0)]:
        b = rng.integers(0, 256, size=(97, bb), dtype=np.uint8)
        want = np.empty(97 * per, dtype=np.float32)
        fn(b.ctypes.data_as(C.c_void_p), want.ctypes.data_as(C.c_void_p), 97)
        got = oracle.dequant(b, qt)
        assert np.array_equal(np.nan_to_num(got).view(np.uint32), np.nan_to_num(want).view(np.uint32))
