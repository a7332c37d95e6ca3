"""Batched prefill on the tensor cores (jinf_b200_prefill_gemm: tcgen05.mma, TMEM accumulator,
TMA-loaded fp16 activations) against a float64 numpy contraction of the exactly dequantised
Q4_0 weights (the reference's dequant, oracle restatement) and the same fp16 inputs.

The weights enter the tensor cores as fp16 products (q - 8) * d, rounded once (relative
error <= 2^-11 per weight); the bar is the per-kernel 1e-3 (max|diff| / max|ref|)."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

REL = 1e-3


def q4_0_rows(rows, cols, seed, std=0.02):
    import jinf
    x = (np.random.default_rng(seed).standard_normal(rows * cols) * std).astype(np.float32)
    out = np.empty(rows * cols // 32 * 18, dtype=np.uint8)
    jinf.lib.jinf_quantize_q4_0(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), rows * cols)
    return out.reshape(rows, -1)


def rel_err(got, want):
    return float(np.max(np.abs(np.asarray(got, np.float64) - want)) / max(np.max(np.abs(want)), 1e-30))


@pytest.mark.parametrize("rows,cols,T", [(6144, 4096, 512), (4096, 4096, 128), (1024, 4096, 100), (37, 1408, 200),
                                         (4096, 14336, 96), (160, 384, 1)])
def test_prefill_gemm_matches_float64(cuda, rows, cols, T):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=rows * 7 + cols)
    q = torch.empty(K.q4m_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    K.q4m_pack(torch.from_numpy(w).to(cuda), q, rows, cols)
    rng = np.random.default_rng(T)
    x = (rng.standard_normal((T, cols)) * 3).astype(np.float16)
    scale = np.exp2(rng.integers(-6, 6, size=T)).astype(np.float32)
    y = torch.full((T, rows), float("nan"), dtype=torch.float32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    K.prefill_gemm(q, rows, cols, torch.from_numpy(x).to(cuda), torch.from_numpy(scale).to(cuda), y, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    wd = oracle.dequant(w.reshape(-1), 2).reshape(rows, cols).astype(np.float64)
    want = (x.astype(np.float64) @ wd.T) * scale[:, None].astype(np.float64)
    got = y.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert rel_err(got, want) < REL


def test_prefill_gemm_deterministic(cuda):
    from jinf import kernels as K
    rows, cols, T = 4096, 4096, 256
    w = q4_0_rows(rows, cols, seed=3)
    q = torch.empty(K.q4m_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    K.q4m_pack(torch.from_numpy(w).to(cuda), q, rows, cols)
    x = torch.from_numpy(np.random.default_rng(1).standard_normal((T, cols)).astype(np.float16)).to(cuda)
    s = torch.ones(T, dtype=torch.float32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    a = torch.empty((T, rows), dtype=torch.float32, device=cuda)
    b = torch.empty_like(a)
    K.prefill_gemm(q, rows, cols, x, s, a, err)
    K.prefill_gemm(q, rows, cols, x, s, b, err)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and int(err.item()) == 0
