"""ctypes access to the CPU oracle (liboracle.so) and to the reference's own host code
compiled from its source tree (_ref/libjinf_ref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs as the checker or the timed CPU baseline. The product
package never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
SYNTH_SO = os.path.join(HERE, "libsynth.so")
REF_SO = os.path.join(HERE, "_ref", "libjinf_ref.so")

_orc = None
_ref = None
_syn = None


def reference_dir() -> str | None:
    """The reference source tree, if this machine has it: $JINF_REFERENCE_DIR, else a
    checkout named `reference` beside this repository. None on machines without it (the
    prebuilt _ref/ files are used there)."""
    cand = os.environ.get("JINF_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isfile(os.path.join(cand, "src", "quant.cpp")) else None


def build() -> None:
    """Build liboracle.so and libsynth.so (and _ref/ when the reference tree is present)."""
    ref = reference_dir()
    cmd = ["make", "-C", HERE] + ([f"REF={ref}"] if ref else [])
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL)


def lib() -> C.CDLL:
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            build()
        o = C.CDLL(ORACLE_SO)
        vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "orc_fp16_to_fp32": (f32, [C.c_uint16]),
            "orc_fp16_to_fp32_array": (None, [vp, vp, i64]),
            "orc_dequant_q4_0": (None, [vp, vp, i64]),
            "orc_dequant_q4_K": (None, [vp, vp, i64]),
            "orc_dequant_q8_0": (None, [vp, vp, i64]),
            "orc_dequant_q6_K": (None, [vp, vp, i64]),
            "orc_matvec": (None, [vp, i32, vp, vp, i32, i32]),
            "orc_rmsnorm": (None, [vp, vp, vp, i32, f32]),
            "orc_rope": (None, [vp, vp, i32, i32, i32, i32, f32]),
            "orc_silu_mul": (None, [vp, vp, vp, i32]),
            "orc_softmax": (None, [vp, vp, i32]),
            "orc_attention": (None, [vp, vp, vp, vp, i32, i32, i32, i32]),
            "orc_sparse_ffn": (None, [vp, vp, vp, vp, i32, i32, i32, vp]),
            "orc_model_create": (vp, [i32, i32, i32, i32, i32, i32, f32, f32, i32, i32]),
            "orc_model_destroy": (None, [vp]),
            "orc_model_bind": (i32, [vp, C.c_char_p, i32, vp]),
            "orc_model_pos": (i32, [vp]),
            "orc_model_set_ffn_mask": (i32, [vp, i32, vp, i32]),
            "orc_forward": (i32, [vp, i32, vp]),
            "orc_argmax": (i32, [vp, i32]),
            "orc_fill_kv_random": (i32, [vp, i32, C.c_uint64]),
            "orc_model_load_kv_f16": (i32, [vp, i32, vp, vp]),
            "orc_num_threads": (i32, []),
        }
        for n, (r, a) in sig.items():
            fn = getattr(o, n)
            fn.restype, fn.argtypes = r, a
        _orc = o
    return _orc


def ref_lib() -> C.CDLL | None:
    """The reference's own quant.cpp / gguf.cpp / splitter.cpp, or None if not built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            if reference_dir():
                build()
            if not os.path.exists(REF_SO):
                return None
        r = C.CDLL(REF_SO)
        vp = C.c_void_p
        for n in ["ref_dequantize_q4_0", "ref_dequantize_q4_K", "ref_dequantize_q8_0"]:
            getattr(r, n).restype, getattr(r, n).argtypes = None, [vp, vp, C.c_int]
        r.ref_dequantize.restype, r.ref_dequantize.argtypes = None, [vp, C.c_int, vp, C.c_longlong]
        r.ref_gguf_summary.restype, r.ref_gguf_summary.argtypes = C.c_int, [C.c_char_p, C.c_char_p, C.c_int]
        r.ref_split.restype = C.c_int
        r.ref_split.argtypes = [C.c_char_p, C.c_ulonglong, C.POINTER(C.c_int), C.POINTER(C.c_ulonglong)]
        _ref = r
    return _ref


def _vp(a: np.ndarray) -> C.c_void_p:
    return a.ctypes.data_as(C.c_void_p)


BLOCK = {2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def dequant(blocks: np.ndarray, qtype: int) -> np.ndarray:
    be, bb = BLOCK[qtype]
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = blocks.size // bb
    out = np.empty(nb * be, dtype=np.float32)
    fn = {2: "orc_dequant_q4_0", 8: "orc_dequant_q8_0", 12: "orc_dequant_q4_K", 14: "orc_dequant_q6_K"}[qtype]
    getattr(lib(), fn)(_vp(blocks), _vp(out), nb)
    return out


def fp16_to_fp32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.size, dtype=np.float32)
    lib().orc_fp16_to_fp32_array(_vp(h), _vp(out), h.size)
    return out


def matvec(w: np.ndarray, qtype: int, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    lib().orc_matvec(_vp(w), qtype, _vp(x), _vp(y), rows, cols)
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_vp(out), _vp(x), _vp(w), x.size, eps)
    return out


def rope(q: np.ndarray, k: np.ndarray, hd: int, nh: int, nkv: int, pos: int, base: float):
    q = np.array(q, dtype=np.float32)
    k = np.array(k, dtype=np.float32)
    lib().orc_rope(_vp(q), _vp(k), hd, nh, nkv, pos, base)
    return q, k


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    lib().orc_silu_mul(_vp(out), _vp(g), _vp(u), g.size)
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_softmax(_vp(out), _vp(x), x.size)
    return out


def attention(q, kc, vc, hd, nh, nkv, n_past) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(kc, dtype=np.float32)
    vc = np.ascontiguousarray(vc, dtype=np.float32)
    out = np.empty(nh * hd, dtype=np.float32)
    lib().orc_attention(_vp(out), _vp(q), _vp(kc), _vp(vc), hd, nh, nkv, n_past)
    return out


def sparse_ffn(bundles, x, offsets, n_act, hidden, qtype) -> tuple[np.ndarray, np.ndarray]:
    bundles = np.ascontiguousarray(bundles, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    offsets = np.ascontiguousarray(offsets, dtype=np.int32)
    out = np.empty(hidden, dtype=np.float32)
    gu = np.empty(max(1, n_act), dtype=np.float32)
    lib().orc_sparse_ffn(_vp(bundles), _vp(x), _vp(out), _vp(offsets), n_act, hidden, qtype, _vp(gu))
    return out, gu[:n_act]


class _HParams(C.Structure):
    _fields_ = [("arch", C.c_char * 64), ("n_layers", C.c_uint32), ("n_embd", C.c_uint32),
                ("n_heads", C.c_uint32), ("n_heads_kv", C.c_uint32), ("n_ff", C.c_uint32),
                ("n_vocab", C.c_uint32), ("n_ctx_train", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rms_norm_eps", C.c_float)]


class _SynthConfig(C.Structure):
    _fields_ = [("hp", _HParams), ("seed", C.c_uint64), ("weight_type", C.c_int),
                ("weight_std", C.c_float), ("embed_std", C.c_float), ("mix_type", C.c_int)]


def synth_lib() -> C.CDLL:
    """libsynth.so: the seeded synthetic-model generator built from the package's generator
    sources, so that CPU baselines and fixture scripts run without the product library."""
    global _syn
    if _syn is None:
        if not os.path.exists(SYNTH_SO):
            build()
        s = C.CDLL(SYNTH_SO)
        vp, i32, i64 = C.c_void_p, C.c_int, C.c_int64
        sig = {
            "jinf_synth_create": (i32, [C.POINTER(vp), C.POINTER(_SynthConfig)]),
            "jinf_synth_destroy": (None, [vp]),
            "jinf_synth_n_tensors": (i32, [vp]),
            "jinf_synth_tensor_name": (C.c_char_p, [vp, i32]),
            "jinf_synth_tensor_info": (i32, [vp, C.c_char_p, C.POINTER(i32), C.POINTER(i64), C.POINTER(i32),
                                             C.POINTER(C.c_uint64)]),
            "jinf_synth_read_rows": (i32, [vp, C.c_char_p, i64, i64, vp]),
            "jinf_synth_write_gguf": (i32, [vp, C.c_char_p]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(s, n)
            fn.restype, fn.argtypes = r, a
        _syn = s
    return _syn


class SynthSource:
    """The seeded synthetic model (same bytes as the package's SynthModel: one generator
    source), read through libsynth.so. `shape` is any object with the LlamaShape fields."""

    def __init__(self, shape, seed: int = 0, weight_type: int = 2, mix_type: int = 0,
                 weight_std: float = 0.02, embed_std: float = 0.02):
        cfg = _SynthConfig()
        cfg.hp.arch = b"llama"
        cfg.hp.n_layers, cfg.hp.n_embd, cfg.hp.n_heads = shape.n_layers, shape.n_embd, shape.n_heads
        cfg.hp.n_heads_kv, cfg.hp.n_ff, cfg.hp.n_vocab = shape.n_heads_kv, shape.n_ff, shape.n_vocab
        cfg.hp.n_ctx_train = getattr(shape, "n_ctx_train", 8192)
        cfg.hp.rope_freq_base, cfg.hp.rms_norm_eps = shape.rope_freq_base, shape.rms_norm_eps
        cfg.seed, cfg.weight_type, cfg.weight_std, cfg.embed_std = seed, weight_type, weight_std, embed_std
        cfg.mix_type = mix_type
        h = C.c_void_p()
        if synth_lib().jinf_synth_create(C.byref(h), C.byref(cfg)) != 0:
            raise RuntimeError("jinf_synth_create failed")
        self.handle, self.shape = h, shape

    def close(self) -> None:
        if self.handle:
            synth_lib().jinf_synth_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor_names(self) -> list[str]:
        n = synth_lib().jinf_synth_n_tensors(self.handle)
        return [synth_lib().jinf_synth_tensor_name(self.handle, i).decode() for i in range(n)]

    def tensor_info(self, name: str):
        t, nd, nb = C.c_int(), C.c_int(), C.c_uint64()
        shape = (C.c_int64 * 4)()
        if synth_lib().jinf_synth_tensor_info(self.handle, name.encode(), C.byref(t), shape, C.byref(nd),
                                              C.byref(nb)) != 0:
            raise KeyError(name)
        return t.value, tuple(shape[i] for i in range(nd.value)), nb.value

    def read_rows(self, name: str, row0: int = 0, n_rows: int | None = None) -> np.ndarray:
        t, shape, nbytes = self.tensor_info(name)
        rows = shape[1] if len(shape) > 1 else 1
        if n_rows is None:
            n_rows = rows - row0
        row_bytes = nbytes // rows
        buf = np.empty(n_rows * row_bytes, dtype=np.uint8)
        if synth_lib().jinf_synth_read_rows(self.handle, name.encode(), row0, n_rows, _vp(buf)) != 0:
            raise RuntimeError(f"read_rows({name})")
        if t == 0:
            return buf.view(np.float32).reshape(n_rows, -1)
        return buf.reshape(n_rows, row_bytes)

    def write_gguf(self, path: str) -> None:
        if synth_lib().jinf_synth_write_gguf(self.handle, path.encode()) != 0:
            raise RuntimeError("write_gguf failed")


class OracleModel:
    """The whole decode step on the CPU, over tensors of a jinf SynthModel (borrowed arrays)."""

    def __init__(self, synth, max_ctx: int, kv_f16: bool = True, layers: int | None = None):
        sh = synth.shape
        self.shape = sh
        self.n_layers = sh.n_layers if layers is None else layers
        o = lib()
        self.h = o.orc_model_create(self.n_layers, sh.n_embd, sh.n_heads, sh.n_heads_kv, sh.n_ff, sh.n_vocab,
                                    sh.rms_norm_eps, sh.rope_freq_base, max_ctx, 1 if kv_f16 else 0)
        self._keep = []
        for name in synth.tensor_names():
            if name.startswith("blk.") and int(name.split(".")[1]) >= self.n_layers:
                continue
            t, _, _ = synth.tensor_info(name)
            arr = np.ascontiguousarray(synth.read_rows(name))
            self._keep.append(arr)
            o.orc_model_bind(self.h, name.encode(), t, _vp(arr))

    def close(self):
        if self.h:
            lib().orc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self) -> int:
        return lib().orc_model_pos(self.h)

    def forward(self, token: int, want_logits: bool = True) -> np.ndarray | None:
        logits = np.empty(self.shape.n_vocab, dtype=np.float32) if want_logits else None
        rc = lib().orc_forward(self.h, int(token), _vp(logits) if want_logits else None)
        if rc != 0:
            raise RuntimeError(f"orc_forward failed ({rc})")
        return logits

    def set_ffn_mask(self, layer: int, ids) -> None:
        """Restrict layer `layer`'s FFN to the neurons `ids` (None: dense)."""
        if ids is None:
            rc = lib().orc_model_set_ffn_mask(self.h, layer, None, -1)
        else:
            a = np.ascontiguousarray(ids, dtype=np.int32)
            rc = lib().orc_model_set_ffn_mask(self.h, layer, _vp(a), int(a.size))
        if rc != 0:
            raise RuntimeError("orc_model_set_ffn_mask failed")

    def fill_kv_random(self, n_pos: int, seed: int = 0) -> None:
        if lib().orc_fill_kv_random(self.h, n_pos, seed) != 0:
            raise RuntimeError("orc_fill_kv_random failed")

    def load_kv_f16(self, k: np.ndarray, v: np.ndarray) -> None:
        """Cache positions [0, n) from fp16 arrays [layers][kv heads][n][head_dim] (the B200
        engine's order, e.g. Engine.kv_read), and set the position to n."""
        k = np.ascontiguousarray(k, dtype=np.float16)
        v = np.ascontiguousarray(v, dtype=np.float16)
        if k.shape != v.shape or k.ndim != 4:
            raise ValueError("k and v must be [layers][kv heads][n][head_dim]")
        if lib().orc_model_load_kv_f16(self.h, k.shape[2], _vp(k), _vp(v)) != 0:
            raise RuntimeError("orc_model_load_kv_f16 failed")


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().orc_argmax(_vp(v), v.size))


def num_threads() -> int:
    return int(lib().orc_num_threads())
