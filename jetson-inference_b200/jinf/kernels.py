"""Thin wrappers of the reference kernel ABI (jinf_cuda_*) and the new B200 entry points
(jinf_b200_*) over torch CUDA tensors: torch provides device memory and the stream, the
computation is the library's."""
from __future__ import annotations

import ctypes as C

from . import _lib as L


def _p(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _s(stream=None) -> C.c_void_p:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _raise_last(what: str) -> None:
    err = L.lib.jinf_cuda_last_error()
    if err:
        raise L.JinfError(err, what)


def dequant_matvec(weight, x, y, rows: int, cols: int, qtype: int, stream=None) -> None:
    L.lib.jinf_cuda_dequant_matvec(_p(weight), _p(x), _p(y), rows, cols, qtype, _s(stream))
    _raise_last("jinf_cuda_dequant_matvec")


def dequantize(blocks, out, n_blocks: int, qtype: int, stream=None) -> None:
    fn = {L.Q4_0: L.lib.jinf_cuda_dequantize_q4_0, L.Q4_K: L.lib.jinf_cuda_dequantize_q4_K,
          L.Q8_0: L.lib.jinf_cuda_dequantize_q8_0, L.Q6_K: L.lib.jinf_cuda_dequantize_q6_K}[qtype]
    fn(_p(blocks), _p(out), n_blocks, _s(stream))
    _raise_last("jinf_cuda_dequantize")


def rmsnorm(out, x, w, n: int, eps: float, weight_type: int = 0, stream=None) -> None:
    L.lib.jinf_cuda_rmsnorm(_p(out), _p(x), _p(w), n, eps, weight_type, _s(stream))
    _raise_last("jinf_cuda_rmsnorm")


def rope(q, k, head_dim: int, n_heads: int, n_heads_kv: int, pos: int, base: float, stream=None) -> None:
    L.lib.jinf_cuda_rope(_p(q), _p(k), head_dim, n_heads, n_heads_kv, pos, base, _s(stream))
    _raise_last("jinf_cuda_rope")


def silu_mul(out, g, u, n: int, stream=None) -> None:
    L.lib.jinf_cuda_silu_mul(_p(out), _p(g), _p(u), n, _s(stream))
    _raise_last("jinf_cuda_silu_mul")


def softmax(out, x, n: int, stream=None) -> None:
    L.lib.jinf_cuda_softmax(_p(out), _p(x), n, _s(stream))
    _raise_last("jinf_cuda_softmax")


def residual_add(a, b, n: int, stream=None) -> None:
    L.lib.jinf_cuda_residual_add(_p(a), _p(b), n, _s(stream))
    _raise_last("jinf_cuda_residual_add")


def attention(out, q, kc, vc, head_dim: int, n_heads: int, n_heads_kv: int, n_past: int, max_ctx: int,
              stream=None) -> None:
    L.lib.jinf_cuda_attention(_p(out), _p(q), _p(kc), _p(vc), head_dim, n_heads, n_heads_kv, n_past, max_ctx,
                              _s(stream))
    _raise_last("jinf_cuda_attention")


def sparse_ffn(bundles, x, out, offsets, n_act: int, hidden: int, bundle_size: int, qtype: int, gate_up,
               stream=None) -> None:
    L.lib.jinf_cuda_sparse_ffn(_p(bundles), _p(x), _p(out), _p(offsets), n_act, hidden, bundle_size, qtype,
                               _p(gate_up), _s(stream))
    _raise_last("jinf_cuda_sparse_ffn")


def q4m_bytes(rows: int, cols: int) -> int:
    return int(L.lib.jinf_b200_q4m_bytes(rows, cols))


def q4m_pack(aos, q4m, rows: int, cols: int, stream=None) -> None:
    L.check(L.lib.jinf_b200_q4m_pack(_p(aos), _p(q4m), rows, cols, _s(stream)), "jinf_b200_q4m_pack")


def gemv_q4m_batch_workspace_bytes(rows: int, cols: int, batch: int) -> int:
    return int(L.lib.jinf_b200_gemv_q4m_batch_workspace_bytes(rows, cols, batch))


def gemv_q4m_batch(q4m, x, y, rows: int, cols: int, batch: int, workspace=None, stream=None) -> None:
    """Y[b] = W . X[b] for the `batch` rows of X ([batch][cols], fp32 or fp16) -> y [batch][rows]."""
    import torch
    xt = L.F32 if x.dtype == torch.float32 else L.F16
    ws = _p(workspace) if workspace is not None else None
    L.check(L.lib.jinf_b200_gemv_q4m_batch(_p(q4m), _p(x), xt, _p(y), rows, cols, batch, ws, _s(stream)),
            "jinf_b200_gemv_q4m_batch")


def gemv_q4m_batch_workspace_bytes_qt(rows: int, cols: int, batch: int, qtype: int) -> int:
    return int(L.lib.jinf_b200_gemv_q4m_batch_workspace_bytes_qt(rows, cols, batch, qtype))


def gemv_q4m_batch_qt(q4m, qtype: int, x, y, rows: int, cols: int, batch: int, workspace=None, kw: int = 0,
                      stream=None) -> None:
    """Y[b] = W . X[b] over a Q4M image of block type `qtype`; kw = 0 picks the K split."""
    import torch
    xt = L.F32 if x.dtype == torch.float32 else L.F16
    ws = _p(workspace) if workspace is not None else None
    L.check(L.lib.jinf_b200_gemv_q4m_batch_qt(_p(q4m), qtype, _p(x), xt, _p(y), rows, cols, batch, ws, kw,
                                              _s(stream)), "jinf_b200_gemv_q4m_batch_qt")


def q4m_bytes_qt(rows: int, cols: int, qtype: int) -> int:
    """Q4M image bytes for qtype Q4_0 (2), Q8_0 (8), Q4_K (12) or Q6_K (14); 0 for an
    unsupported type or shape."""
    return int(L.lib.jinf_b200_q4m_bytes_qt(rows, cols, qtype))


def q4m_pack_qt(aos, qtype: int, q4m, rows: int, cols: int, stream=None) -> None:
    L.check(L.lib.jinf_b200_q4m_pack_qt(_p(aos), qtype, _p(q4m), rows, cols, _s(stream)), "jinf_b200_q4m_pack_qt")


def gemv_q4m_qt(q4m, qtype: int, x, y, rows: int, cols: int, workspace=None, kw: int = 0, stream=None) -> None:
    import torch
    xt = L.F32 if x.dtype == torch.float32 else L.F16
    ws = _p(workspace) if workspace is not None else None
    L.check(L.lib.jinf_b200_gemv_q4m_qt(_p(q4m), qtype, _p(x), xt, _p(y), rows, cols, ws, kw, _s(stream)),
            "jinf_b200_gemv_q4m_qt")


def gemv_q4m_workspace_bytes(rows: int, cols: int) -> int:
    return int(L.lib.jinf_b200_gemv_q4m_workspace_bytes(rows, cols))


def gemv_q4m(q4m, x, y, rows: int, cols: int, workspace=None, kw: int = 0, stream=None) -> None:
    """kw = 0 picks the K split for the device; kw > 1 needs a zeroed workspace tensor."""
    import torch
    xt = L.F32 if x.dtype == torch.float32 else L.F16
    ws = _p(workspace) if workspace is not None else None
    L.check(L.lib.jinf_b200_gemv_q4m(_p(q4m), _p(x), xt, _p(y), rows, cols, ws, kw, _s(stream)),
            "jinf_b200_gemv_q4m")


def gemv_q4m_rmsnorm(q4m, h, gain, eps: float, y, rows: int, cols: int, workspace=None, kw: int = 0,
                     stream=None) -> None:
    ws = _p(workspace) if workspace is not None else None
    L.check(L.lib.jinf_b200_gemv_q4m_rmsnorm(_p(q4m), _p(h), _p(gain), eps, _p(y), rows, cols, ws, kw,
                                             _s(stream)), "jinf_b200_gemv_q4m_rmsnorm")


def attention_workspace_bytes(n_kv_heads: int, head_dim: int, max_ctx: int) -> int:
    return int(L.lib.jinf_b200_attention_workspace_bytes(n_kv_heads, head_dim, max_ctx))


def attention_f16(out, q, kc, vc, head_dim: int, n_heads: int, n_kv_heads: int, n_pos: int, max_ctx: int,
                  workspace, stream=None) -> None:
    L.check(L.lib.jinf_b200_attention_f16(_p(out), _p(q), _p(kc), _p(vc), head_dim, n_heads, n_kv_heads, n_pos,
                                          max_ctx, _p(workspace), _s(stream)), "jinf_b200_attention_f16")


def prefill_gemm(q4m, rows: int, cols: int, x16, tok_scale, y, err, accumulate: bool = False, stream=None) -> None:
    """y[t][m] (+)= tok_scale[t] * sum_k x16[t][k] W[m][k] over the T rows of x16 ([T][cols] fp16):
    the tensor-core (tcgen05) contraction of the batched prefill. `err`: a zeroed device int32."""
    T = int(x16.shape[0])
    L.check(L.lib.jinf_b200_prefill_gemm(_p(q4m), rows, cols, _p(x16), T, _p(tok_scale), _p(y), int(y.shape[1]),
                                         1 if accumulate else 0, _p(err), _s(stream)), "jinf_b200_prefill_gemm")
