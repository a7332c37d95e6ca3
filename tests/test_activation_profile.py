"""Activation profiles in the reference's static-predictor format (writer: reference
tools/profile_activations.cpp:143-162; reader and the frequency > threshold rule: reference
src/activation_predictor.cpp:226-300), and the calibration prompt generator. CPU only."""
import ctypes as C

import numpy as np
import pytest


def ref_profile_bytes(counts: np.ndarray, total: int) -> bytes:
    """The file as the reference tool writes it: int32 n_layers, n_ff, total_tokens, then the
    float32 frequencies count / total per layer."""
    n_layers, n_ff = counts.shape
    hdr = np.array([n_layers, n_ff, total], dtype=np.int32).tobytes()
    freq = (counts.astype(np.float32) / np.float32(total)) if total > 0 else np.zeros(counts.shape, np.float32)
    return hdr + freq.astype(np.float32).tobytes()


@pytest.fixture(scope="module")
def lib():
    import jinf
    return jinf.lib


def test_profile_write_matches_reference_bytes(lib, tmp_path):
    rng = np.random.default_rng(3)
    counts = rng.integers(0, 500, size=(4, 1408)).astype(np.int32)
    path = tmp_path / "act.bin"
    assert lib.jinf_activation_profile_write(str(path).encode(), 4, 1408, 500, counts.ctypes.data) == 0
    assert path.read_bytes() == ref_profile_bytes(counts, 500)


@pytest.mark.parametrize("thr", [0.0, 0.25, 0.5, 0.99])
def test_profile_read_applies_the_static_rule(lib, tmp_path, thr):
    rng = np.random.default_rng(int(thr * 100))
    freq = rng.random((3, 256)).astype(np.float32)
    freq[0, :7] = thr  # equal to the threshold: not active (strictly greater)
    path = tmp_path / "act.bin"
    path.write_bytes(np.array([3, 256, 1000], np.int32).tobytes() + freq.tobytes())
    ids = np.full((3, 256), -1, np.int32)
    n = np.zeros(3, np.int32)
    assert lib.jinf_activation_profile_read(str(path).encode(), C.c_float(thr), 3, 256, ids.ctypes.data,
                                            n.ctypes.data) == 0
    for l in range(3):
        want = np.nonzero(freq[l] > np.float32(thr))[0]
        assert n[l] == len(want)
        assert np.array_equal(ids[l, :n[l]], want)


def test_profile_read_rejects_other_shapes_and_truncation(lib, tmp_path):
    from jinf import _lib as L
    freq = np.zeros((2, 64), np.float32)
    path = tmp_path / "act.bin"
    path.write_bytes(np.array([2, 64, 10], np.int32).tobytes() + freq.tobytes())
    ids = np.zeros(2 * 128, np.int32)
    n = np.zeros(2, np.int32)
    assert lib.jinf_activation_profile_read(str(path).encode(), C.c_float(0.5), 2, 128, ids.ctypes.data,
                                            n.ctypes.data) == L.JINF_ERR_INVALID
    path.write_bytes(np.array([2, 64, 10], np.int32).tobytes() + freq.tobytes()[:100])
    assert lib.jinf_activation_profile_read(str(path).encode(), C.c_float(0.5), 2, 64, ids.ctypes.data,
                                            n.ctypes.data) == L.JINF_ERR_PARSE
    assert lib.jinf_activation_profile_read(str(tmp_path / "missing.bin").encode(), C.c_float(0.5), 2, 64,
                                            ids.ctypes.data, n.ctypes.data) == L.JINF_ERR_IO


def test_calibration_prompts_follow_the_reference_generator():
    """srand(42); each prompt 8 + rand() % 24 tokens of rand() % n_vocab, in that order."""
    from jinf.calibrate import reference_prompts
    libc = C.CDLL(None)
    libc.rand.restype = C.c_int
    libc.srand(42)
    want = []
    for _ in range(3):
        n = 8 + libc.rand() % 24
        want.append([libc.rand() % 4096 for _ in range(n)])
    got = list(reference_prompts(3, 4096))
    assert got == want
    assert all(8 <= len(p) < 32 for p in got)
