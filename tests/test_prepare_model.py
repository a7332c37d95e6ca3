"""GGUF -> NVMW conversion (jinf_prepare_model) against the reference's own
tools/prepare_model: the file is identical byte for byte, pinned by the committed hashes of
the reference's output (tests/golden/make_prepare_golden.py) and, where the reference tool
was built here (oracle/_ref/prepare_model), by running it side by side. CPU only."""
import ctypes as C
import hashlib
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "prepare_model_ref.txt")
REF_TOOL = os.path.join(ROOT, "oracle", "_ref", "prepare_model")


def golden_cases():
    out = []
    for ln in open(GOLDEN):
        if ln.startswith("#") or not ln.strip():
            continue
        budget, bundled, size, digest = ln.split()
        out.append((int(budget), int(bundled), int(size), digest))
    return out


@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory):
    import jinf
    path = str(tmp_path_factory.mktemp("prep") / "tiny.gguf")
    jinf.SynthModel(jinf.TINY, seed=0).write_gguf(path)
    return path


def prepare(gguf, out, budget, bundled):
    import jinf
    assert jinf.lib.jinf_prepare_model(gguf.encode(), out.encode(), budget, bundled) == 0


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: f"budget{c[0]}_bundled{c[1]}")
def test_prepare_matches_reference_hash(tiny_gguf, tmp_path, case):
    budget, bundled, size, digest = case
    out = str(tmp_path / "ours.nvmw")
    prepare(tiny_gguf, out, budget, bundled)
    data = open(out, "rb").read()
    assert len(data) == size
    assert hashlib.sha256(data).hexdigest() == digest


@pytest.mark.skipif(not os.path.exists(REF_TOOL), reason="reference prepare_model not built here")
def test_prepare_matches_reference_tool_side_by_side(tiny_gguf, tmp_path):
    ref, ours = str(tmp_path / "ref.nvmw"), str(tmp_path / "ours.nvmw")
    subprocess.run([REF_TOOL, "--input", tiny_gguf, "--output", ref, "--gpu-budget", "64", "--bundled"], check=True,
                   capture_output=True)
    prepare(tiny_gguf, ours, 64, 1)
    assert open(ref, "rb").read() == open(ours, "rb").read()


def test_prepared_file_reads_back(tiny_gguf, tmp_path):
    """Our NVMW reader opens the converted (bundled) file: every tensor's bytes at its file
    offset equal the synthetic model's, and the bundle index is found."""
    import jinf
    lib = jinf.lib
    out = str(tmp_path / "ours.nvmw")
    prepare(tiny_gguf, out, 8, 1)
    syn = jinf.SynthModel(jinf.TINY, seed=0)
    r = C.c_void_p()
    assert lib.jinf_nvmw_open(C.byref(r), out.encode()) == 0
    try:
        assert lib.jinf_nvmw_has_bundles(r)
        for name in ("blk.1.ffn_down.weight", "blk.3.attn_q.weight", "output.weight"):
            te = lib.jinf_nvmw_find_tensor(r, name.encode())
            assert te
            want = syn.read_rows(name).tobytes()
            with open(out, "rb") as f:
                f.seek(lib.jinf_nvmw_tensor_file_offset(r, C.cast(te, C.c_void_p)))
                assert f.read(len(want)) == want
    finally:
        lib.jinf_nvmw_close(r)
