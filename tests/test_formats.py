"""Loader formats and the engine's error contract on the CPU (no GPU needed).

Mirrors the reference's own tests: tests/test_gguf.cpp (minimal GGUF v3 parse),
tests/test_splitter.cpp (always-hot set, huge budget, promotion order),
tests/test_engine.cpp (config defaults, invalid path, null arguments); and checks this
library's GGUF writer + reader and splitter against golden output of the reference's
own parser and splitter (tests/golden/gguf_split_ref.txt).
"""
import ctypes as C
import os
import struct

import numpy as np
import pytest

import jinf
from jinf import _lib as L

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "gguf_split_ref.txt")


def _gguf_str(s: bytes) -> bytes:
    return struct.pack("<Q", len(s)) + s


def write_reference_test_gguf(path):
    """The file of reference tests/test_gguf.cpp:35-78: 5 KVs, one Q4_0 tensor [64, 100]."""
    b = struct.pack("<IIQQ", 0x46554747, 3, 1, 5)
    b += _gguf_str(b"general.architecture") + struct.pack("<I", 8) + _gguf_str(b"llama")
    b += _gguf_str(b"llama.block_count") + struct.pack("<II", 4, 2)
    b += _gguf_str(b"llama.embedding_length") + struct.pack("<II", 4, 64)
    b += _gguf_str(b"llama.attention.head_count") + struct.pack("<II", 4, 4)
    b += _gguf_str(b"llama.attention.layer_norm_rms_epsilon") + struct.pack("<If", 6, 1e-5)
    b += _gguf_str(b"token_embd.weight") + struct.pack("<IqqIQ", 2, 64, 100, 2, 0)
    b += b"\0" * ((32 - len(b) % 32) % 32)
    b += b"\0" * (64 * 100 // 32 * 18)
    open(path, "wb").write(b)


def test_gguf_reference_fixture(tmp_path):
    p = str(tmp_path / "t.gguf")
    write_reference_test_gguf(p)
    f = C.POINTER(L.GgufFile)()
    assert L.lib.jinf_gguf_open(C.byref(f), p.encode()) == 0
    g = f.contents
    assert (g.version, g.tensor_count, g.kv_count) == (3, 1, 5)
    hp = g.hparams
    assert (hp.n_layers, hp.n_embd, hp.n_heads, hp.arch) == (2, 64, 4, b"llama")
    assert hp.n_heads_kv == 4  # defaults to n_heads
    kv = L.lib.jinf_gguf_find_kv(f, b"llama.block_count")
    assert kv and kv.contents.u32 == 2
    assert L.lib.jinf_gguf_get_u32(f, b"llama.embedding_length", 0) == 64
    t = g.tensor_infos[0]
    assert (t.n_dims, t.shape[0], t.shape[1], t.type, t.n_elements) == (2, 64, 100, jinf.Q4_0, 6400)
    assert L.lib.jinf_gguf_find_tensor(f, b"token_embd.weight").contents.shape[0] == 64
    assert not L.lib.jinf_gguf_find_kv(f, b"nonexistent")
    assert not L.lib.jinf_gguf_find_tensor(f, b"nonexistent")
    L.lib.jinf_gguf_close(f)
    bad = C.POINTER(L.GgufFile)()
    assert L.lib.jinf_gguf_open(C.byref(bad), b"/nonexistent/file.gguf") != 0
    assert not bad


@pytest.mark.parametrize("corrupt", ["magic", "version", "truncated"])
def test_gguf_corrupt_files(tmp_path, corrupt):
    p = str(tmp_path / "t.gguf")
    write_reference_test_gguf(p)
    data = bytearray(open(p, "rb").read())
    if corrupt == "magic":
        data[0] ^= 0xFF
    elif corrupt == "version":
        data[4] = 9
    else:
        data = data[:60]
    open(p, "wb").write(bytes(data))
    f = C.POINTER(L.GgufFile)()
    assert L.lib.jinf_gguf_open(C.byref(f), p.encode()) == L.JINF_ERR_PARSE
    assert not f


def _golden_lines():
    return open(GOLD).read().splitlines()


def test_gguf_writer_reader_match_reference_parser(tmp_path):
    """Our writer's file, parsed by our reader, gives exactly what the reference parser gave."""
    shape = jinf.LlamaShape(2, 256, 4, 2, 512, 1024, 10000.0, 1e-5)
    m = jinf.SynthModel(shape, seed=7)
    p = str(tmp_path / "m.gguf")
    m.write_gguf(p)
    f = C.POINTER(L.GgufFile)()
    assert L.lib.jinf_gguf_open(C.byref(f), p.encode()) == 0
    g = f.contents
    lines = [f"status 0 {g.version} {g.tensor_count} {g.kv_count} {g.alignment} {g.data_offset}"]
    h = g.hparams
    lines.append("hp %s %u %u %u %u %u %u %u %.9g %.9g" % (h.arch.decode(), h.n_layers, h.n_embd, h.n_heads,
                                                          h.n_heads_kv, h.n_ff, h.n_vocab, h.n_ctx_train,
                                                          h.rope_freq_base, h.rms_norm_eps))
    for i in range(g.tensor_count):
        t = g.tensor_infos[i]
        lines.append(f"t {t.name.decode()} {t.n_dims} {t.shape[0]} {t.shape[1]} {t.type} {t.offset} "
                     f"{t.n_elements} {t.n_bytes}")
    gold = [ln for ln in _golden_lines() if not ln.startswith("split")]
    assert lines == gold
    # splitter placements vs the reference splitter on the same file
    for ln in _golden_lines():
        if not ln.startswith("split"):
            continue
        _, budget, cnt, hot, cold, pl = ln.split()
        cfg = L.SplitConfig(int(budget), 0, 0)
        plan = C.POINTER(L.SplitPlan)()
        assert L.lib.jinf_split_analyze(f, C.byref(cfg), C.byref(plan)) == 0
        got = "".join(str(plan.contents.assignments[i].placement) for i in range(plan.contents.count))
        assert (plan.contents.count, plan.contents.total_hot_bytes, plan.contents.total_cold_bytes, got) == \
            (int(cnt), int(hot), int(cold), pl)
        L.lib.jinf_split_plan_free(plan)
    L.lib.jinf_gguf_close(f)


def _splitter_model(n_layers):
    """The in-memory model of reference tests/test_splitter.cpp:13-74 (Q4_K, Llama-7B-like)."""
    names = [("token_embd.weight", 4096, 32000, jinf.Q4_K), ("output.weight", 4096, 32000, jinf.Q4_K),
             ("output_norm.weight", 4096, 1, jinf.F32)]
    for l in range(n_layers):
        names += [(f"blk.{l}.attn_norm.weight", 4096, 1, jinf.F32), (f"blk.{l}.ffn_norm.weight", 4096, 1, jinf.F32),
                  (f"blk.{l}.attn_q.weight", 4096, 4096, jinf.Q4_K), (f"blk.{l}.attn_k.weight", 1024, 4096, jinf.Q4_K),
                  (f"blk.{l}.attn_v.weight", 1024, 4096, jinf.Q4_K),
                  (f"blk.{l}.attn_output.weight", 4096, 4096, jinf.Q4_K),
                  (f"blk.{l}.ffn_gate.weight", 11008, 4096, jinf.Q4_K),
                  (f"blk.{l}.ffn_up.weight", 11008, 4096, jinf.Q4_K),
                  (f"blk.{l}.ffn_down.weight", 4096, 11008, jinf.Q4_K)]
    infos = (L.GgufTensorInfo * len(names))()
    keep = []
    for i, (n, r, c, t) in enumerate(names):
        nb = n.encode()
        keep.append(nb)
        infos[i].name = nb
        infos[i].n_dims = 2
        infos[i].shape[0], infos[i].shape[1] = r, c
        infos[i].type = t
        infos[i].n_elements = r * c
        be, bb = L.BLOCK_ELEMS[t], L.BLOCK_BYTES[t]
        infos[i].n_bytes = (r * c + be - 1) // be * bb
    g = L.GgufFile()
    g.hparams.n_layers, g.hparams.n_embd, g.hparams.n_ff = n_layers, 4096, 11008
    g.tensor_count = len(names)
    g.tensor_infos = C.cast(infos, C.POINTER(L.GgufTensorInfo))
    return g, infos, keep


def _plan(g, budget):
    cfg = L.SplitConfig(budget, 0, 0)
    plan = C.POINTER(L.SplitPlan)()
    assert L.lib.jinf_split_analyze(C.byref(g), C.byref(cfg), C.byref(plan)) == 0
    return plan


def test_splitter_always_hot():
    g, infos, keep = _splitter_model(2)
    plan = _plan(g, 0)
    hot = [plan.contents.assignments[i].tensor.contents.name.decode() for i in range(plan.contents.count)
           if plan.contents.assignments[i].placement == 0]
    assert len(hot) == 7
    assert all(("embd" in n) or ("output" in n) or ("norm" in n) for n in hot)
    L.lib.jinf_split_plan_free(plan)


def test_splitter_large_budget():
    g, infos, keep = _splitter_model(2)
    plan = _plan(g, 100 << 30)
    assert all(plan.contents.assignments[i].placement == 0 for i in range(plan.contents.count))
    assert plan.contents.total_cold_bytes == 0
    L.lib.jinf_split_plan_free(plan)


def test_splitter_promotion_order():
    g, infos, keep = _splitter_model(4)
    p0 = _plan(g, 0)
    always = p0.contents.total_hot_bytes
    L.lib.jinf_split_plan_free(p0)
    attn = (4096 * 4096 + 1024 * 4096 * 2 + 4096 * 4096) // 256 * 144
    plan = _plan(g, always + attn + 1024)
    for i in range(plan.contents.count):
        a = plan.contents.assignments[i]
        name = a.tensor.contents.name.decode()
        if a.layer_index == 0 and "attn_" in name and "norm" not in name:
            assert a.placement == 0
        if a.layer_index == 1 and "attn_q" in name:
            assert a.placement == 1
    L.lib.jinf_split_plan_free(plan)


def test_tp_roles():
    roles = {"blk.3.attn_q.weight": 1, "blk.3.attn_k.weight": 1, "blk.3.attn_v.weight": 1,
             "blk.3.attn_output.weight": 2, "blk.3.ffn_gate.weight": 1, "blk.3.ffn_up.weight": 1,
             "blk.3.ffn_down.weight": 2, "output.weight": 1, "token_embd.weight": 0, "blk.0.attn_norm.weight": 0}
    for n, r in roles.items():
        assert L.lib.jinf_split_tp_role(n.encode()) == r, n


def test_nvmw_roundtrip(tmp_path):
    shape = jinf.LlamaShape(2, 256, 4, 2, 512, 1024, 10000.0, 1e-5)
    m = jinf.SynthModel(shape, seed=3)
    p = str(tmp_path / "m.nvmw")
    m.write_nvmw(p)
    r = C.c_void_p()
    assert L.lib.jinf_nvmw_open(C.byref(r), p.encode()) == 0
    h = L.lib.jinf_nvmw_get_header(r).contents
    assert (h.magic, h.version, h.n_layers, h.n_embd, h.n_heads, h.n_heads_kv, h.n_ff, h.n_vocab) == \
        (0x574D564E, 1, 2, 256, 4, 2, 512, 1024)
    assert h.hot_offset % 4096 == 0 and h.primary_type == jinf.Q4_0
    n = C.c_int()
    ents = L.lib.jinf_nvmw_get_tensor_entries(r, C.byref(n))
    assert n.value == len(m.tensor_names())
    raw = open(p, "rb").read()
    for i in range(n.value):
        e = ents[i]
        name = e.name.decode()
        off = L.lib.jinf_nvmw_tensor_file_offset(r, C.byref(e))
        assert off % 4096 == 0
        want = m.read_rows(name).tobytes()
        assert raw[off:off + e.n_bytes] == want, name
        assert e.layer_index == (int(name.split(".")[1]) if name.startswith("blk.") else -1)
    assert not L.lib.jinf_nvmw_has_bundles(r)
    L.lib.jinf_nvmw_close(r)


def test_nvmw_bad_magic_and_missing(tmp_path):
    p = str(tmp_path / "bad.nvmw")
    open(p, "wb").write(b"\0" * 8192)
    r = C.c_void_p()
    assert L.lib.jinf_nvmw_open(C.byref(r), p.encode()) == L.JINF_ERR_PARSE
    assert L.lib.jinf_nvmw_open(C.byref(r), b"/nonexistent.nvmw") == L.JINF_ERR_IO


# ---- engine error contract (reference tests/test_engine.cpp:14-63) -------------------------

def test_engine_config_defaults():
    # jinf_engine_config_default() is a header inline; mirror its values through the struct
    cfg = L.EngineConfig()
    cfg.gpu_memory_budget, cfg.buffer_capacity, cfg.max_context, cfg.io_queue_depth = 4500 << 20, 128 << 20, 512, 64
    assert cfg.model_path is None and cfg.gpu_memory_budget > 0 and cfg.max_context > 0


def test_engine_invalid_model_path():
    cfg = L.EngineConfig()
    cfg.model_path = b"/tmp/nonexistent_model.nvmw"
    cfg.max_context = 512
    e = C.POINTER(L.Engine)()
    assert L.lib.jinf_engine_create(C.byref(e), C.byref(cfg)) != 0
    assert not e


def test_engine_null_arguments():
    cfg = L.EngineConfig()
    e = C.POINTER(L.Engine)()
    assert L.lib.jinf_engine_create(None, None) == L.JINF_ERR_INVALID
    assert L.lib.jinf_engine_create(None, C.byref(cfg)) == L.JINF_ERR_INVALID
    assert L.lib.jinf_engine_create(C.byref(e), None) == L.JINF_ERR_INVALID
    tok = (C.c_int32 * 1)(1)
    logits = C.c_void_p()
    assert L.lib.jinf_engine_forward(None, tok, 1, C.byref(logits)) == L.JINF_ERR_INVALID
    out = (C.c_int32 * 4)()
    n = C.c_int()
    assert L.lib.jinf_engine_generate(None, tok, 1, out, 4, C.byref(n)) == L.JINF_ERR_INVALID
    assert not L.lib.jinf_engine_get_stats(None)
    L.lib.jinf_engine_reset(None)
    L.lib.jinf_engine_destroy(None)
