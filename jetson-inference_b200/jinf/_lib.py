"""ctypes binding of libjinf_b200.so (the C-ABI declared in include/jinf/*.h).

The shared library is built in-tree (``make -C jetson-inference_b200``) and loaded
from next to this package. There is no fallback: if the library is missing the import
fails loudly, because every compute path of this package runs on the GPU through it.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
# JINF_LIB selects another build of the same library (e.g. a tuning variant)
LIB_PATH = os.environ.get("JINF_LIB") or os.path.join(PKG_ROOT, "libjinf_b200.so")

# jinf_status values (include/jinf/common.h)
JINF_OK, JINF_ERR_IO, JINF_ERR_PARSE, JINF_ERR_CUDA, JINF_ERR_OOM, JINF_ERR_INVALID, JINF_ERR_TIMEOUT = range(7)
STATUS_NAMES = {0: "OK", 1: "I/O error", 2: "parse error", 3: "CUDA error", 4: "out of memory",
                5: "invalid argument", 6: "timed out"}

# jinf_qtype values (include/jinf/quant.h)
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
BLOCK_ELEMS = {F32: 1, F16: 1, Q4_0: 32, Q8_0: 32, Q4_K: 256, Q6_K: 256}
BLOCK_BYTES = {F32: 4, F16: 2, Q4_0: 18, Q8_0: 34, Q4_K: 144, Q6_K: 210}


class JinfError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)} ({status})")
        self.status = status


class HParams(C.Structure):
    _fields_ = [("arch", C.c_char * 64), ("n_layers", C.c_uint32), ("n_embd", C.c_uint32),
                ("n_heads", C.c_uint32), ("n_heads_kv", C.c_uint32), ("n_ff", C.c_uint32),
                ("n_vocab", C.c_uint32), ("n_ctx_train", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rms_norm_eps", C.c_float)]


class SynthConfig(C.Structure):
    _fields_ = [("hp", HParams), ("seed", C.c_uint64), ("weight_type", C.c_int),
                ("weight_std", C.c_float), ("embed_std", C.c_float), ("mix_type", C.c_int)]


class EngineConfig(C.Structure):
    _fields_ = [("model_path", C.c_char_p), ("gpu_memory_budget", C.c_size_t), ("buffer_capacity", C.c_size_t),
                ("max_context", C.c_int), ("io_queue_depth", C.c_int), ("predictor_path", C.c_char_p),
                ("sparsity_threshold", C.c_float)]


class B200Options(C.Structure):
    _fields_ = [("device", C.c_int), ("tp_rank", C.c_int), ("tp_size", C.c_int), ("nccl_id", C.c_void_p),
                ("kv_type", C.c_int), ("use_graph", C.c_int), ("eos_token", C.c_int), ("sparse_mode", C.c_int),
                ("sparse_keep", C.c_float), ("sparse_seed", C.c_uint64), ("persistent", C.c_int), ("prefill", C.c_int),
                ("max_seqs", C.c_int)]


class PerfStats(C.Structure):
    _fields_ = [("total_ms", C.c_double), ("nvme_read_ms", C.c_double), ("gpu_compute_ms", C.c_double),
                ("attention_ms", C.c_double), ("ffn_ms", C.c_double), ("tokens_generated", C.c_int),
                ("nvme_bytes_read", C.c_double)]


FFN_HOOK = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_void_p, C.c_int)


class Engine(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_embd", C.c_int), ("n_heads", C.c_int), ("n_heads_kv", C.c_int),
                ("n_ff", C.c_int), ("n_vocab", C.c_int), ("max_context", C.c_int), ("head_dim", C.c_int),
                ("rms_norm_eps", C.c_float), ("rope_freq_base", C.c_float), ("primary_type", C.c_int32),
                ("n_past", C.c_int), ("ffn_hook", FFN_HOOK), ("ffn_hook_data", C.c_void_p),
                ("logits_buf", C.c_void_p), ("compute_stream", C.c_void_p), ("perf", PerfStats),
                ("impl", C.c_void_p)]


class GgufTensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", C.c_uint32), ("shape", C.c_int64 * 4), ("type", C.c_int),
                ("offset", C.c_uint64), ("n_elements", C.c_int64), ("n_bytes", C.c_size_t)]


class GgufKV(C.Structure):
    class _V(C.Union):
        _fields_ = [("u32", C.c_uint32), ("i32", C.c_int32), ("f32", C.c_float), ("u64", C.c_uint64),
                    ("f64", C.c_double), ("str", C.c_char_p * 2), ("raw", C.c_uint8 * 24)]
    _anonymous_ = ("v",)
    _fields_ = [("key", C.c_char_p), ("type", C.c_int), ("v", _V)]


class GgufFile(C.Structure):
    _fields_ = [("version", C.c_uint32), ("tensor_count", C.c_uint64), ("kv_count", C.c_uint64),
                ("alignment", C.c_uint32), ("kvs", C.POINTER(GgufKV)), ("tensor_infos", C.POINTER(GgufTensorInfo)),
                ("data_offset", C.c_size_t), ("hparams", HParams)]


class SplitConfig(C.Structure):
    _fields_ = [("gpu_memory_budget", C.c_size_t), ("kv_cache_budget", C.c_size_t), ("buffer_budget", C.c_size_t)]


class WeightAssignment(C.Structure):
    _fields_ = [("tensor", C.POINTER(GgufTensorInfo)), ("placement", C.c_int), ("layer_index", C.c_int)]


class SplitPlan(C.Structure):
    _fields_ = [("assignments", C.POINTER(WeightAssignment)), ("count", C.c_int),
                ("total_hot_bytes", C.c_size_t), ("total_cold_bytes", C.c_size_t)]


class NvmwHeader(C.Structure):
    _pack_ = 1
    _fields_ = [("magic", C.c_uint32), ("version", C.c_uint32), ("n_layers", C.c_uint32), ("n_tensors", C.c_uint32),
                ("index_offset", C.c_uint64), ("index_size", C.c_uint64), ("hot_offset", C.c_uint64),
                ("hot_size", C.c_uint64), ("cold_start_offset", C.c_uint64), ("cold_total_size", C.c_uint64),
                ("n_embd", C.c_uint32), ("n_heads", C.c_uint32), ("n_heads_kv", C.c_uint32), ("n_ff", C.c_uint32),
                ("n_vocab", C.c_uint32), ("n_ctx_train", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rms_norm_eps", C.c_float), ("primary_type", C.c_int32), ("_pad0", C.c_uint32),
                ("bundle_index_offset", C.c_uint64), ("_reserved", C.c_uint8 * (4096 - 112))]


class NvmwTensorEntry(C.Structure):
    _fields_ = [("name", C.c_char * 128), ("type", C.c_int), ("shape", C.c_int64 * 4), ("n_dims", C.c_uint32),
                ("offset", C.c_uint64), ("n_bytes", C.c_uint64), ("layer_index", C.c_int32), ("is_hot", C.c_uint8),
                ("_pad", C.c_uint8 * 3)]


vp, i32, i64, u64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float, C.c_size_t

# name -> (restype, argtypes); every function declared in include/jinf/*.h
SIGNATURES = {
    # quant.h
    "jinf_dequantize_q4_0": (None, [vp, vp, i32]),
    "jinf_dequantize_q4_K": (None, [vp, vp, i32]),
    "jinf_dequantize_q8_0": (None, [vp, vp, i32]),
    "jinf_dequantize_q6_K": (None, [vp, vp, i32]),
    "jinf_dequantize": (None, [vp, i32, vp, i64]),
    "jinf_fp16_to_fp32": (f32, [C.c_uint16]),
    "jinf_fp32_to_fp16": (C.c_uint16, [f32]),
    "jinf_quantize_q4_0": (None, [vp, vp, i64]),
    "jinf_quantize_q4_K": (None, [vp, vp, i64]),
    "jinf_quantize_q8_0": (None, [vp, vp, i64]),
    "jinf_b200_q4m_pack_host": (i32, [vp, i32, vp, i32, i32]),
    "jinf_quantize_q6_K": (None, [vp, vp, i64]),
    # kernels.h
    "jinf_cuda_dequant_matvec": (None, [vp, vp, vp, i32, i32, i32, vp]),
    "jinf_cuda_residual_add": (None, [vp, vp, i32, vp]),
    "jinf_cuda_dequantize_q4_0": (None, [vp, vp, i32, vp]),
    "jinf_cuda_dequantize_q4_K": (None, [vp, vp, i32, vp]),
    "jinf_cuda_dequantize_q8_0": (None, [vp, vp, i32, vp]),
    "jinf_cuda_dequantize_q6_K": (None, [vp, vp, i32, vp]),
    "jinf_cuda_rmsnorm": (None, [vp, vp, vp, i32, f32, i32, vp]),
    "jinf_cuda_rope": (None, [vp, vp, i32, i32, i32, i32, f32, vp]),
    "jinf_cuda_silu_mul": (None, [vp, vp, vp, i32, vp]),
    "jinf_cuda_softmax": (None, [vp, vp, i32, vp]),
    "jinf_cuda_attention": (None, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "jinf_cuda_last_error": (i32, []),
    # sparse_ops.h
    "jinf_cuda_sparse_ffn": (None, [vp, vp, vp, vp, i32, i32, i32, i32, vp, vp]),
    # b200.h
    "jinf_b200_q4m_bytes": (u64, [i32, i32]),
    "jinf_b200_q4m_pack": (i32, [vp, vp, i32, i32, vp]),
    "jinf_b200_q4m_bytes_qt": (u64, [i32, i32, i32]),
    "jinf_b200_gemv_q4m_batch_workspace_bytes": (sz, [i32, i32, i32]),
    "jinf_b200_gemv_q4m_batch": (i32, [vp, vp, i32, vp, i32, i32, i32, vp, vp]),
    "jinf_b200_gemv_q4m_batch_workspace_bytes_qt": (sz, [i32, i32, i32, i32]),
    "jinf_b200_gemv_q4m_batch_qt": (i32, [vp, i32, vp, i32, vp, i32, i32, i32, vp, i32, vp]),
    "jinf_b200_q4m_pack_qt": (i32, [vp, i32, vp, i32, i32, vp]),
    "jinf_b200_gemv_q4m_qt": (i32, [vp, i32, vp, i32, vp, i32, i32, vp, i32, vp]),
    "jinf_b200_gemv_q4m_workspace_bytes": (sz, [i32, i32]),
    "jinf_b200_gemv_q4m": (i32, [vp, vp, i32, vp, i32, i32, vp, i32, vp]),
    "jinf_b200_gemv_q4m_rmsnorm": (i32, [vp, vp, vp, f32, vp, i32, i32, vp, i32, vp]),
    "jinf_b200_gemv_q4m_noalloc": (i32, [vp, vp, i32, vp, i32, i32, vp]),
    "jinf_b200_prefill_gemm": (i32, [vp, i32, i32, vp, i32, vp, vp, i32, i32, vp, vp]),
    "jinf_b200_attention_workspace_bytes": (sz, [i32, i32, i32]),
    "jinf_b200_attention_f16": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp]),
    # gguf.h
    "jinf_gguf_open": (i32, [C.POINTER(C.POINTER(GgufFile)), C.c_char_p]),
    "jinf_gguf_close": (None, [C.POINTER(GgufFile)]),
    "jinf_gguf_find_kv": (C.POINTER(GgufKV), [C.POINTER(GgufFile), C.c_char_p]),
    "jinf_gguf_find_tensor": (C.POINTER(GgufTensorInfo), [C.POINTER(GgufFile), C.c_char_p]),
    "jinf_gguf_get_str": (C.c_char_p, [C.POINTER(GgufFile), C.c_char_p, C.c_char_p]),
    "jinf_gguf_get_u32": (C.c_uint32, [C.POINTER(GgufFile), C.c_char_p, C.c_uint32]),
    "jinf_gguf_get_f32": (f32, [C.POINTER(GgufFile), C.c_char_p, f32]),
    "jinf_gguf_writer_create": (i32, [C.POINTER(vp), C.c_char_p]),
    "jinf_gguf_writer_add_kv_u32": (i32, [vp, C.c_char_p, C.c_uint32]),
    "jinf_gguf_writer_add_kv_f32": (i32, [vp, C.c_char_p, f32]),
    "jinf_gguf_writer_add_kv_str": (i32, [vp, C.c_char_p, C.c_char_p]),
    "jinf_gguf_writer_add_tensor": (i32, [vp, C.c_char_p, i32, C.POINTER(C.c_int64), i32, vp, sz]),
    "jinf_gguf_writer_finish": (i32, [vp]),
    # nvmw.h
    "jinf_nvmw_writer_create": (i32, [C.POINTER(vp), C.c_char_p]),
    "jinf_nvmw_writer_destroy": (None, [vp]),
    "jinf_nvmw_writer_set_header": (i32, [vp, C.POINTER(NvmwHeader)]),
    "jinf_nvmw_writer_add_layer_desc": (i32, [vp, i32, vp]),
    "jinf_nvmw_writer_add_tensor_entry": (i32, [vp, C.POINTER(NvmwTensorEntry)]),
    "jinf_nvmw_writer_write_hot": (i32, [vp, vp, sz]),
    "jinf_nvmw_writer_write_cold_layer": (i32, [vp, i32, vp, sz]),
    "jinf_nvmw_writer_finalize": (i32, [vp]),
    "jinf_nvmw_writer_write_bundle_section": (i32, [vp, vp, vp, i32]),
    "jinf_prepare_model": (i32, [C.c_char_p, C.c_char_p, sz, i32]),
    "jinf_prepare_model_b200": (i32, [C.c_char_p, C.c_char_p]),
    "jinf_prepare_model_b200_tp": (i32, [C.c_char_p, C.c_char_p, i32]),
    "jinf_nvmw_open": (i32, [C.POINTER(vp), C.c_char_p]),
    "jinf_nvmw_close": (None, [vp]),
    "jinf_nvmw_get_header": (C.POINTER(NvmwHeader), [vp]),
    "jinf_nvmw_get_layer_desc": (vp, [vp, i32]),
    "jinf_nvmw_get_tensor_entries": (C.POINTER(NvmwTensorEntry), [vp, C.POINTER(i32)]),
    "jinf_nvmw_get_layer_cold_range": (i32, [vp, i32, C.POINTER(u64), C.POINTER(u64)]),
    "jinf_nvmw_get_hot_range": (i32, [vp, C.POINTER(u64), C.POINTER(u64)]),
    "jinf_nvmw_find_tensor": (C.POINTER(NvmwTensorEntry), [vp, C.c_char_p]),
    "jinf_nvmw_has_bundles": (C.c_bool, [vp]),
    "jinf_nvmw_get_bundle_header": (vp, [vp]),
    "jinf_nvmw_get_bundle_layer_desc": (vp, [vp, i32]),
    "jinf_nvmw_get_neuron_bundle_offset": (u64, [vp, i32, i32]),
    "jinf_nvmw_tensor_file_offset": (u64, [vp, vp]),
    "jinf_nvmw_get_path": (C.c_char_p, [vp]),
    # splitter.h
    "jinf_split_analyze": (i32, [C.POINTER(GgufFile), C.POINTER(SplitConfig), C.POINTER(C.POINTER(SplitPlan))]),
    "jinf_split_plan_free": (None, [C.POINTER(SplitPlan)]),
    "jinf_split_plan_print": (None, [C.POINTER(SplitPlan)]),
    "jinf_split_tp_role": (i32, [C.c_char_p]),
    "jinf_tp_shard": (i32, [C.c_char_p, C.c_int64, C.c_int64, i32, i32, vp, vp, vp, vp]),
    # engine.h
    "jinf_engine_create": (i32, [C.POINTER(C.POINTER(Engine)), C.POINTER(EngineConfig)]),
    "jinf_engine_destroy": (None, [C.POINTER(Engine)]),
    "jinf_engine_forward": (i32, [C.POINTER(Engine), C.POINTER(C.c_int32), i32, C.POINTER(C.c_void_p)]),
    "jinf_engine_generate": (i32, [C.POINTER(Engine), C.POINTER(C.c_int32), i32, C.POINTER(C.c_int32), i32,
                                   C.POINTER(i32)]),
    "jinf_engine_reset": (None, [C.POINTER(Engine)]),
    "jinf_engine_get_stats": (C.POINTER(PerfStats), [C.POINTER(Engine)]),
    "jinf_engine_create_ex": (i32, [C.POINTER(C.POINTER(Engine)), C.POINTER(EngineConfig), C.POINTER(B200Options)]),
    "jinf_engine_create_synthetic": (i32, [C.POINTER(C.POINTER(Engine)), C.POINTER(EngineConfig), vp,
                                           C.POINTER(B200Options)]),
    "jinf_engine_decode_resident": (i32, [C.POINTER(Engine), i32, C.POINTER(C.c_int32)]),
    "jinf_engine_last_argmax": (i32, [C.POINTER(Engine), C.POINTER(C.c_int32)]),
    "jinf_engine_fill_kv_random": (i32, [C.POINTER(Engine), i32, u64]),
    "jinf_engine_kv_read": (i32, [C.POINTER(Engine), i32, vp, vp]),
    "jinf_engine_decode_batch": (i32, [C.POINTER(Engine), i32, vp, vp, vp, vp]),
    "jinf_engine_decode_batch_resident": (i32, [C.POINTER(Engine), i32, vp, vp, i32, vp]),
    "jinf_engine_seq_n_past": (i32, [C.POINTER(Engine), i32]),
    "jinf_engine_seq_reset": (i32, [C.POINTER(Engine), i32]),
    "jinf_engine_seq_fill_kv_random": (i32, [C.POINTER(Engine), i32, i32, u64]),
    "jinf_engine_seq_kv_read": (i32, [C.POINTER(Engine), i32, i32, vp, vp]),
    "jinf_engine_is_persistent": (i32, [vp]),
    "jinf_engine_sparse_ids": (i32, [vp, i32, vp, i32, vp]),
    "jinf_engine_count_activations": (i32, [vp, vp, i32, C.c_float, vp]),
    "jinf_engine_debug_step_timeout": (i32, [vp, C.c_ulonglong]),
    "jinf_activation_profile_write": (i32, [C.c_char_p, i32, i32, i32, vp]),
    "jinf_activation_profile_read": (i32, [C.c_char_p, C.c_float, i32, i32, vp, vp]),
    "jinf_sparse_fixed_mask": (i32, [C.c_uint64, i32, i32, C.c_float, vp]),
    "jinf_sparse_predictor_weights": (None, [C.c_uint64, i32, i32, i64, vp]),
    "jinf_b200_sparse_predict": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, vp, vp, vp, vp]),
    "jinf_engine_weight_bytes_per_token": (u64, [C.POINTER(Engine)]),
    "jinf_engine_profile_kernels": (i32, [C.POINTER(Engine), i32, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "jinf_engine_profile_multi": (i32, [C.POINTER(Engine), i32, i32, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "jinf_nccl_get_unique_id": (i32, [vp]),
    "jinf_synth_create": (i32, [C.POINTER(vp), C.POINTER(SynthConfig)]),
    "jinf_synth_destroy": (None, [vp]),
    "jinf_synth_get_config": (C.POINTER(SynthConfig), [vp]),
    "jinf_synth_n_tensors": (i32, [vp]),
    "jinf_synth_tensor_name": (C.c_char_p, [vp, i32]),
    "jinf_synth_tensor_info": (i32, [vp, C.c_char_p, C.POINTER(i32), C.POINTER(C.c_int64), C.POINTER(i32),
                                     C.POINTER(u64)]),
    "jinf_synth_read_rows": (i32, [vp, C.c_char_p, i64, i64, vp]),
    "jinf_synth_read_rows_device": (i32, [vp, C.c_char_p, i64, i64, vp, vp]),
    "jinf_synth_write_gguf": (i32, [vp, C.c_char_p]),
    "jinf_synth_write_nvmw": (i32, [vp, C.c_char_p]),
}


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {PKG_ROOT}` "
                          "(the CUDA library is required; there is no fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status: int, what: str = "jinf call") -> None:
    if status != JINF_OK:
        raise JinfError(status, what)
