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


def test_prepare_b200_layout_holds_engine_images(tmp_path):
    """jinf_prepare_model_b200 (new, no reference counterpart): a version-3 file whose
    projections are the engine's fused Q4M images. Checked against the numpy restatement of
    the layout: gate|up interleaved by neuron, and a v of its own type (Q6_K in the even
    layers of a Q4_K_M-like model) kept apart from [q | k]."""
    import numpy as np
    import jinf
    import q4m_ref
    from jinf import _lib as L
    shape = jinf.LlamaShape(2, 512, 8, 2, 1536, 1024, 10000.0, 1e-5)
    syn = jinf.SynthModel(shape, seed=5, weight_type=L.Q4_K, mix_type=L.Q6_K)
    gguf = str(tmp_path / "m.gguf")
    out = str(tmp_path / "m.nvmw")
    syn.write_gguf(gguf)
    assert L.lib.jinf_prepare_model_b200(gguf.encode(), out.encode()) == 0
    r = C.c_void_p()
    assert L.lib.jinf_nvmw_open(C.byref(r), out.encode()) == 0
    try:
        h = L.lib.jinf_nvmw_get_header(r).contents
        assert h.version == 3
        raw = np.fromfile(out, dtype=np.uint8)

        def image(name):
            e = L.lib.jinf_nvmw_find_tensor(r, name.encode())
            assert e, name
            e = e.contents
            o = h.hot_offset + e.offset
            return e.type, (e.shape[1], e.shape[0]), raw[o:o + e.n_bytes]

        names = {L.lib.jinf_nvmw_get_tensor_entries(r, C.byref(C.c_int()))[i].name.decode()
                 for i in range(h.n_tensors)}
        assert "blk.0.v.q4m" in names and "blk.1.v.q4m" not in names   # v in Q6_K only in even layers
        t, (rows, cols), img = image("blk.0.v.q4m")
        assert t == 0x40 + 2 and (rows, cols) == (128, 512)
        assert np.array_equal(img, q4m_ref.pack_q6k(syn.read_rows("blk.0.attn_v.weight"), rows, cols))
        t, (rows, cols), img = image("blk.1.gu.q4m")
        assert t == 0x40 + 1 and (rows, cols) == (2 * 1536, 512)
        g, u = syn.read_rows("blk.1.ffn_gate.weight"), syn.read_rows("blk.1.ffn_up.weight")
        inter = np.empty((2 * g.shape[0], g.shape[1]), dtype=np.uint8)
        inter[0::2], inter[1::2] = g, u
        assert np.array_equal(img, q4m_ref.pack_q4k(inter, rows, cols))
        t, (rows, cols), img = image("output.q4m")
        assert t == 0x40 + 2 and (rows, cols) == (1024, 512)
        t, _, _ = image("blk.1.qkv.q4m")
        assert t == 0x40 + 1
    finally:
        L.lib.jinf_nvmw_close(r)


@pytest.mark.parametrize("tp", [2, 4])
def test_prepare_b200_tp_shards(tmp_path, tp):
    """jinf_prepare_model_b200_tp: every rank's slice of every projection as its own image
    ("tp<N>.<rank>." + the one-GPU name), in the engine's split: q, k, v, gate, up and the output
    head by rows (heads / neurons / vocabulary), o and down by whole column blocks. Each image
    equals the numpy packing of the rank's slice of the source blocks."""
    import numpy as np
    import jinf
    import q4m_ref
    from jinf import _lib as L
    shape = jinf.LlamaShape(2, 1024, 16, 4, 2048, 1024, 10000.0, 1e-5)
    syn = jinf.SynthModel(shape, seed=6, weight_type=L.Q4_K, mix_type=L.Q6_K)
    gguf = str(tmp_path / "m.gguf")
    out = str(tmp_path / "m.nvmw")
    syn.write_gguf(gguf)
    assert L.lib.jinf_prepare_model_b200_tp(gguf.encode(), out.encode(), tp) == 0
    assert L.lib.jinf_prepare_model_b200_tp(gguf.encode(), out.encode(), 3) != 0
    r = C.c_void_p()
    assert L.lib.jinf_nvmw_open(C.byref(r), out.encode()) == 0
    try:
        h = L.lib.jinf_nvmw_get_header(r).contents
        raw = np.fromfile(out, dtype=np.uint8)

        def image(name):
            e = L.lib.jinf_nvmw_find_tensor(r, name.encode())
            assert e, name
            e = e.contents
            o = h.hot_offset + e.offset
            return e.type, (e.shape[1], e.shape[0]), raw[o:o + e.n_bytes]

        hd = 1024 // 16
        for rank in range(tp):
            pre = f"tp{tp}.{rank}."
            rows = lambda n, total: slice(rank * total // tp, (rank + 1) * total // tp)  # noqa: E731
            # layer 0: v in Q6_K (its own image), q|k fused Q4_K
            q = syn.read_rows("blk.0.attn_q.weight")[rows(0, 16 * hd)]
            k = syn.read_rows("blk.0.attn_k.weight")[rows(0, 4 * hd)]
            t, (nr, nc), img = image(pre + "blk.0.qkv.q4m")
            assert (nr, nc) == (q.shape[0] + k.shape[0], 1024)
            assert np.array_equal(img, q4m_ref.pack_q4k(np.concatenate([q, k]), nr, nc))
            v = syn.read_rows("blk.0.attn_v.weight")[rows(0, 4 * hd)]
            t, (nr, nc), img = image(pre + "blk.0.v.q4m")
            assert t == 0x40 + 2 and np.array_equal(img, q4m_ref.pack_q6k(v, nr, nc))
            # gate|up interleaved over the rank's neurons
            g = syn.read_rows("blk.1.ffn_gate.weight")[rows(0, 2048)]
            u = syn.read_rows("blk.1.ffn_up.weight")[rows(0, 2048)]
            inter = np.empty((2 * g.shape[0], g.shape[1]), dtype=np.uint8)
            inter[0::2], inter[1::2] = g, u
            t, (nr, nc), img = image(pre + "blk.1.gu.q4m")
            assert (nr, nc) == (2 * 2048 // tp, 1024) and np.array_equal(img, q4m_ref.pack_q4k(inter, nr, nc))
            # o: the rank's column blocks (Q4_K super-blocks of 256: 144 bytes each)
            o = syn.read_rows("blk.1.attn_output.weight")
            nb = 1024 // 256 // tp
            t, (nr, nc), img = image(pre + "blk.1.o.q4m")
            cols = o[:, rank * nb * 144:(rank + 1) * nb * 144]
            assert (nr, nc) == (1024, 1024 // tp) and np.array_equal(img, q4m_ref.pack_q4k(cols, nr, nc))
            # down: columns of the rank's neurons (layer 0's down is Q6_K: 210-byte super-blocks)
            nbd = 2048 // 256 // tp
            dn = syn.read_rows("blk.1.ffn_down.weight")
            t, (nr, nc), img = image(pre + "blk.1.down.q4m")
            assert (nr, nc) == (1024, 2048 // tp)
            assert np.array_equal(img, q4m_ref.pack_q4k(dn[:, rank * nbd * 144:(rank + 1) * nbd * 144], nr, nc))
            dn0 = syn.read_rows("blk.0.ffn_down.weight")
            t, (nr, nc), img = image(pre + "blk.0.down.q4m")
            assert t == 0x40 + 2
            assert np.array_equal(img, q4m_ref.pack_q6k(dn0[:, rank * nbd * 210:(rank + 1) * nbd * 210], nr, nc))
            # the output head: the rank's vocabulary rows (Q6_K)
            t, (nr, nc), img = image(pre + "output.q4m")
            outw = syn.read_rows("output.weight")[rows(0, 1024)]
            assert t == 0x40 + 2 and np.array_equal(img, q4m_ref.pack_q6k(outw, nr, nc))
    finally:
        L.lib.jinf_nvmw_close(r)


def test_prepare_b200_tp_refuses_split_blocks(tmp_path):
    """A split that would cut a Q4_K super-block (o of a 512-wide model over 4 GPUs: 128
    columns) is refused."""
    import jinf
    from jinf import _lib as L
    syn = jinf.SynthModel(jinf.LlamaShape(1, 512, 8, 4, 1024, 256, 10000.0, 1e-5), seed=1, weight_type=L.Q4_K)
    gguf = str(tmp_path / "m.gguf")
    syn.write_gguf(gguf)
    assert L.lib.jinf_prepare_model_b200_tp(gguf.encode(), str(tmp_path / "m.nvmw").encode(), 4) != 0
    assert L.lib.jinf_prepare_model_b200_tp(gguf.encode(), str(tmp_path / "m.nvmw").encode(), 2) == 0
