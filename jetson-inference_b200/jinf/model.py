"""Host-side mirror of the reference's engine API (reference include/jinf/engine.h:161-176).

`Engine` wraps jinf_engine_* with the reference's semantics (forward returns device
logits of the last token, generate is greedy with EOS = 2 and first-max argmax);
`SynthModel` wraps the seeded synthetic Llama generator used for every benchmark and
parity configuration.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L


@dataclass
class LlamaShape:
    n_layers: int
    n_embd: int
    n_heads: int
    n_heads_kv: int
    n_ff: int
    n_vocab: int
    rope_freq_base: float = 10000.0
    rms_norm_eps: float = 1e-5
    n_ctx_train: int = 8192

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_heads

    def hparams(self) -> L.HParams:
        h = L.HParams()
        h.arch = b"llama"
        h.n_layers, h.n_embd, h.n_heads = self.n_layers, self.n_embd, self.n_heads
        h.n_heads_kv, h.n_ff, h.n_vocab = self.n_heads_kv, self.n_ff, self.n_vocab
        h.n_ctx_train, h.rope_freq_base, h.rms_norm_eps = self.n_ctx_train, self.rope_freq_base, self.rms_norm_eps
        return h


# BASELINE.json configurations (shapes only; weights come from the seeded generator)
TINY = LlamaShape(4, 512, 8, 2, 1408, 4096, 10000.0, 1e-5)
LLAMA3_8B = LlamaShape(32, 4096, 32, 8, 14336, 128256, 500000.0, 1e-5)
LLAMA3_70B = LlamaShape(80, 8192, 64, 8, 28672, 128256, 500000.0, 1e-5)


class SynthModel:
    """Seeded synthetic model: every value is a pure function of (seed, tensor, index)."""

    def __init__(self, shape: LlamaShape, seed: int = 0, weight_type: int = L.Q4_0,
                 weight_std: float = 0.02, embed_std: float = 0.02, mix_type: int = 0):
        """mix_type (e.g. Q6_K with weight_type Q4_K, a Q4_K_M-like file) is the type of attn_v
        and ffn_down in the even layers and of the output head; 0 keeps one type throughout."""
        cfg = L.SynthConfig()
        cfg.hp = shape.hparams()
        cfg.seed, cfg.weight_type, cfg.weight_std, cfg.embed_std = seed, weight_type, weight_std, embed_std
        cfg.mix_type = mix_type
        h = C.c_void_p()
        L.check(L.lib.jinf_synth_create(C.byref(h), C.byref(cfg)), "jinf_synth_create")
        self.handle = h
        self.shape = shape
        self.seed = seed
        self.weight_type = weight_type
        self.mix_type = mix_type

    def close(self) -> None:
        if self.handle:
            L.lib.jinf_synth_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor_names(self) -> list[str]:
        n = L.lib.jinf_synth_n_tensors(self.handle)
        return [L.lib.jinf_synth_tensor_name(self.handle, i).decode() for i in range(n)]

    def tensor_info(self, name: str) -> tuple[int, tuple[int, ...], int]:
        t, nd, nb = C.c_int(), C.c_int(), C.c_uint64()
        shape = (C.c_int64 * 4)()
        L.check(L.lib.jinf_synth_tensor_info(self.handle, name.encode(), C.byref(t), shape, C.byref(nd),
                                             C.byref(nb)), f"tensor_info({name})")
        return t.value, tuple(shape[i] for i in range(nd.value)), nb.value

    def read_rows(self, name: str, row0: int = 0, n_rows: int | None = None) -> np.ndarray:
        """Rows of a tensor in file layout: uint8 blocks for quantized types, float32 otherwise."""
        t, shape, nbytes = self.tensor_info(name)
        rows = shape[1] if len(shape) > 1 else 1
        if n_rows is None:
            n_rows = rows - row0
        row_bytes = nbytes // rows
        buf = np.empty(n_rows * row_bytes, dtype=np.uint8)
        L.check(L.lib.jinf_synth_read_rows(self.handle, name.encode(), row0, n_rows,
                                           buf.ctypes.data_as(C.c_void_p)), f"read_rows({name})")
        if t == L.F32:
            return buf.view(np.float32).reshape(n_rows, -1)
        return buf.reshape(n_rows, row_bytes)

    def read_rows_device(self, name: str, out, row0: int = 0, n_rows: int | None = None, stream=None):
        """Generate rows on the GPU into the torch tensor `out` (same bytes as read_rows)."""
        import torch
        t, shape, nbytes = self.tensor_info(name)
        rows = shape[1] if len(shape) > 1 else 1
        if n_rows is None:
            n_rows = rows - row0
        if out.numel() * out.element_size() < n_rows * (nbytes // rows):
            raise ValueError("output tensor too small")
        s = stream if stream is not None else torch.cuda.current_stream()
        L.check(L.lib.jinf_synth_read_rows_device(self.handle, name.encode(), row0, n_rows,
                                                  C.c_void_p(out.data_ptr()), C.c_void_p(s.cuda_stream)),
                f"read_rows_device({name})")
        return out

    def write_nvmw(self, path: str) -> None:
        L.check(L.lib.jinf_synth_write_nvmw(self.handle, path.encode()), "write_nvmw")

    def write_gguf(self, path: str) -> None:
        L.check(L.lib.jinf_synth_write_gguf(self.handle, path.encode()), "write_gguf")


def b200_options(device: int = 0, tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None,
                 use_graph: bool = True, eos_token: int = 2, persistent: bool = True, sparse_mode: int = 0,
                 sparse_keep: float = 0.15, sparse_seed: int = 0, prefill: bool = True,
                 max_seqs: int = 1) -> L.B200Options:
    """sparse_mode: 0 dense FFN, 1 device predictor top-k, 2 fixed mask (runs of 8). prefill:
    forward() of several tokens runs all but the last through the batched (tensor-core) prefill
    where the model allows it. max_seqs: sequences with their own KV cache for decode_batch."""
    o = L.B200Options()
    o.device, o.tp_rank, o.tp_size = device, tp_rank, tp_size
    o.kv_type, o.use_graph, o.eos_token = L.F16, int(use_graph), eos_token
    o.sparse_mode, o.sparse_keep, o.sparse_seed = sparse_mode, sparse_keep, sparse_seed
    o.persistent = int(persistent)
    o.prefill = int(prefill)
    o.max_seqs = int(max_seqs)
    o._nccl_buf = None
    if nccl_id is not None:
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        o._nccl_buf = buf  # keep alive
        o.nccl_id = C.cast(buf, C.c_void_p)
    return o


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    L.check(L.lib.jinf_nccl_get_unique_id(buf), "jinf_nccl_get_unique_id")
    return buf.raw


class Engine:
    """jinf_engine_* with the reference's call semantics."""

    def __init__(self, handle):
        self.h = handle

    @classmethod
    def from_nvmw(cls, path: str, max_context: int = 512, options: L.B200Options | None = None,
                  predictor_path: str | None = None, sparsity_threshold: float = 0.5) -> "Engine":
        cfg = L.EngineConfig()
        cfg.model_path = path.encode()
        cfg.gpu_memory_budget, cfg.buffer_capacity = 4500 << 20, 128 << 20
        cfg.max_context, cfg.io_queue_depth, cfg.sparsity_threshold = max_context, 64, sparsity_threshold
        if predictor_path:
            cfg.predictor_path = predictor_path.encode()
        e = C.POINTER(L.Engine)()
        if options is None:
            L.check(L.lib.jinf_engine_create(C.byref(e), C.byref(cfg)), "jinf_engine_create")
        else:
            L.check(L.lib.jinf_engine_create_ex(C.byref(e), C.byref(cfg), C.byref(options)), "jinf_engine_create_ex")
        return cls(e)

    @classmethod
    def from_synth(cls, model: SynthModel, max_context: int = 512,
                   options: L.B200Options | None = None, predictor_path: str | None = None,
                   sparsity_threshold: float = 0.5) -> "Engine":
        """`predictor_path`: an activation profile in the reference's format (static predictor:
        the neurons with frequency > sparsity_threshold run, the FFN in sparse mode)."""
        cfg = L.EngineConfig()
        cfg.max_context, cfg.io_queue_depth, cfg.sparsity_threshold = max_context, 64, sparsity_threshold
        if predictor_path:
            cfg.predictor_path = predictor_path.encode()
        opts = options if options is not None else b200_options()
        e = C.POINTER(L.Engine)()
        L.check(L.lib.jinf_engine_create_synthetic(C.byref(e), C.byref(cfg), model.handle, C.byref(opts)),
                "jinf_engine_create_synthetic")
        return cls(e)

    def close(self) -> None:
        if self.h:
            L.lib.jinf_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def n_past(self) -> int:
        return self.h.contents.n_past

    @property
    def n_vocab(self) -> int:
        return self.h.contents.n_vocab

    def forward(self, tokens) -> int:
        """Run tokens; returns the device pointer of fp32 logits [n_vocab]."""
        arr = (C.c_int32 * len(tokens))(*tokens)
        out = C.c_void_p()
        L.check(L.lib.jinf_engine_forward(self.h, arr, len(tokens), C.byref(out)), "jinf_engine_forward")
        return out.value

    def logits_host(self, tokens) -> np.ndarray:
        """forward() then copy the logits to the host (through torch, the device plumbing)."""
        import torch
        ptr = self.forward(tokens)
        n = self.n_vocab
        host = np.empty(n, dtype=np.float32)
        torch.cuda.synchronize()
        cudart = _cudart()
        rc = cudart.cudaMemcpy(host.ctypes.data_as(C.c_void_p), C.c_void_p(ptr), C.c_size_t(4 * n), 2)
        if rc != 0:
            raise L.JinfError(L.JINF_ERR_CUDA, f"cudaMemcpy {rc}")
        return host

    def generate(self, prompt, max_tokens: int) -> list[int]:
        out = (C.c_int32 * max(1, max_tokens))()
        n = C.c_int(0)
        p = (C.c_int32 * max(1, len(prompt)))(*prompt) if prompt else None
        L.check(L.lib.jinf_engine_generate(self.h, p, len(prompt), out, max_tokens, C.byref(n)), "generate")
        return list(out[: n.value])

    def last_argmax(self) -> int:
        t = C.c_int32()
        L.check(L.lib.jinf_engine_last_argmax(self.h, C.byref(t)), "last_argmax")
        return t.value

    def decode_resident(self, n_steps: int, collect: bool = False) -> list[int] | None:
        buf = (C.c_int32 * max(1, n_steps))() if collect else None
        L.check(L.lib.jinf_engine_decode_resident(self.h, n_steps, buf), "decode_resident")
        return list(buf[:n_steps]) if collect else None

    def reset(self) -> None:
        L.lib.jinf_engine_reset(self.h)

    def fill_kv_random(self, n_pos: int, seed: int = 0) -> None:
        L.check(L.lib.jinf_engine_fill_kv_random(self.h, n_pos, seed), "fill_kv_random")

    def kv_read(self, n_pos: int, tp_size: int = 1):
        """(K, V) of positions [0, n_pos) of this rank's cache as fp16 arrays
        [n_layers][kv heads of this rank][n_pos][head_dim] (tp_size: the engine's ranks)."""
        e = self.h.contents
        hkv = e.n_heads_kv // max(1, tp_size)
        shp = (e.n_layers, hkv, n_pos, e.n_embd // e.n_heads)
        k, v = np.empty(shp, dtype=np.float16), np.empty(shp, dtype=np.float16)
        L.check(L.lib.jinf_engine_kv_read(self.h, n_pos, k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p)),
                "kv_read")
        return k, v

    # ---- multi-sequence decode

    def decode_batch(self, seqs, tokens, want_logits: bool = False):
        """One step of len(seqs) sequences: tokens[i] fed to sequence seqs[i]. Returns the
        greedy next tokens (and the logits [n][n_vocab] when want_logits)."""
        n = len(seqs)
        s = (C.c_int32 * n)(*[int(v) for v in seqs])
        t = (C.c_int32 * n)(*[int(v) for v in tokens])
        out = (C.c_int32 * n)()
        lg = np.empty((n, self.n_vocab), dtype=np.float32) if want_logits else None
        L.check(L.lib.jinf_engine_decode_batch(self.h, n, s, t, out,
                                               lg.ctypes.data_as(C.c_void_p) if want_logits else None),
                "decode_batch")
        return (list(out), lg) if want_logits else list(out)

    def decode_batch_resident(self, seqs, tokens, n_steps: int, collect: bool = False):
        """n_steps greedy steps of the sequences, argmax fed back on the device; returns the
        ids [n_steps][len(seqs)] when collect."""
        n = len(seqs)
        s = (C.c_int32 * n)(*[int(v) for v in seqs])
        t = (C.c_int32 * n)(*[int(v) for v in tokens])
        out = (C.c_int32 * (n * n_steps))() if collect else None
        L.check(L.lib.jinf_engine_decode_batch_resident(self.h, n, s, t, n_steps, out), "decode_batch_resident")
        return [list(out[i * n:(i + 1) * n]) for i in range(n_steps)] if collect else None

    def seq_n_past(self, seq: int) -> int:
        return int(L.lib.jinf_engine_seq_n_past(self.h, seq))

    def seq_reset(self, seq: int) -> None:
        L.check(L.lib.jinf_engine_seq_reset(self.h, seq), "seq_reset")

    def seq_fill_kv_random(self, seq: int, n_pos: int, seed: int = 0) -> None:
        L.check(L.lib.jinf_engine_seq_fill_kv_random(self.h, seq, n_pos, seed), "seq_fill_kv_random")

    def seq_kv_read(self, seq: int, n_pos: int, tp_size: int = 1):
        e = self.h.contents
        hkv = e.n_heads_kv // max(1, tp_size)
        shp = (e.n_layers, hkv, n_pos, e.n_embd // e.n_heads)
        k, v = np.empty(shp, dtype=np.float16), np.empty(shp, dtype=np.float16)
        L.check(L.lib.jinf_engine_seq_kv_read(self.h, seq, n_pos, k.ctypes.data_as(C.c_void_p),
                                              v.ctypes.data_as(C.c_void_p)), "seq_kv_read")
        return k, v

    @property
    def persistent(self) -> bool:
        """True when each decode token runs as one persistent kernel."""
        return bool(L.lib.jinf_engine_is_persistent(self.h))

    def sparse_ids(self, layer: int) -> np.ndarray:
        """Sparse modes: the active neurons of `layer` used by the last forward."""
        n = C.c_int()
        L.check(L.lib.jinf_engine_sparse_ids(self.h, layer, None, 0, C.byref(n)), "jinf_engine_sparse_ids")
        out = np.empty(n.value, dtype=np.int32)
        L.check(L.lib.jinf_engine_sparse_ids(self.h, layer, out.ctypes.data_as(C.c_void_p), n.value, C.byref(n)),
                "jinf_engine_sparse_ids")
        return out

    def count_activations(self, tokens, threshold: float, counts: np.ndarray) -> None:
        """Calibration: forward `tokens`, adding to counts [n_layers, n_ff] (int32) the tokens
        on which |SiLU(gate)| > threshold (reference tools/profile_activations.cpp)."""
        assert counts.dtype == np.int32 and counts.flags.c_contiguous
        arr = np.ascontiguousarray(tokens, dtype=np.int32)
        L.check(L.lib.jinf_engine_count_activations(self.h, arr.ctypes.data_as(C.c_void_p), len(arr), threshold,
                                                    counts.ctypes.data_as(C.c_void_p)), "jinf_engine_count_activations")

    def weight_bytes_per_token(self) -> int:
        return L.lib.jinf_engine_weight_bytes_per_token(self.h)

    def profile_kernels(self, reps: int = 32) -> dict:
        t = (C.c_double * 7)()
        b = (C.c_double * 7)()
        L.check(L.lib.jinf_engine_profile_kernels(self.h, reps, t, b), "profile_kernels")
        names = ["qkv", "attention", "o_proj", "gate_up", "down", "lm_head", "sparse_ffn"]
        return {n: {"us": t[i], "bytes": b[i]} for i, n in enumerate(names)}

    def profile_multi(self, n: int, reps: int = 32) -> dict:
        """Per-kernel times of an n-vector multi-sequence step (the sequences' state is left
        undefined)."""
        t = (C.c_double * 8)()
        b = (C.c_double * 8)()
        L.check(L.lib.jinf_engine_profile_multi(self.h, n, reps, t, b), "profile_multi")
        names = ["qkv", "attention", "o_proj", "gate_up", "down", "lm_head", "rows", "finalize"]
        return {k: {"us": t[i], "bytes": b[i]} for i, k in enumerate(names)}

    def stats(self) -> L.PerfStats:
        return L.lib.jinf_engine_get_stats(self.h).contents


_CUDART = None


def _cudart():
    """The CUDA runtime that torch loaded (device plumbing for host copies in tests)."""
    global _CUDART
    if _CUDART is None:
        import glob
        import os
        import torch  # noqa: F401  (makes sure libcudart is mapped)
        cands = []
        for p in open("/proc/self/maps").read().splitlines():
            if "libcudart.so" in p:
                cands.append(p.split()[-1])
        if not cands:
            base = os.path.dirname(__import__("torch").__file__)
            cands = glob.glob(os.path.join(base, "..", "nvidia", "cuda_runtime", "lib", "libcudart.so*"))
        _CUDART = C.CDLL(cands[0])
        _CUDART.cudaMemcpy.restype = C.c_int
        _CUDART.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    return _CUDART
