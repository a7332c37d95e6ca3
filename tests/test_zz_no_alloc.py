"""jinf_b200_gemv_q4m_noalloc (allocation-free: the split-K workspace is a static device
array inside the library) against jinf_b200_gemv_q4m with a caller workspace and against
the CPU oracle. Collected last, so it also runs after every other GPU test has used the
device; it must pass alone too."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

REL = 1e-3
JINF_OK, JINF_ERR_INVALID = 0, 5  # include/jinf/common.h


def q4_0_rows(rows, cols, seed, std=0.02):
    import jinf
    x = (np.random.default_rng(seed).standard_normal(rows * cols) * std).astype(np.float32)
    out = np.empty(rows * cols // 32 * 18, dtype=np.uint8)
    jinf.lib.jinf_quantize_q4_0(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), rows * cols)
    return out.reshape(rows, -1)


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def noalloc(q, x, y, rows, cols):
    import jinf
    xt = jinf.F32 if x.dtype == torch.float32 else jinf.F16
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return jinf.lib.jinf_b200_gemv_q4m_noalloc(C.c_void_p(q.data_ptr()), C.c_void_p(x.data_ptr()), xt,
                                               C.c_void_p(y.data_ptr()), rows, cols, stream)


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (28672, 4096), (4096, 14336), (37, 384), (1024, 4096),
                                       (128256, 4096)])
def test_noalloc_matches_workspace_gemv_twice(cuda, rows, cols):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=rows ^ cols)
    q = torch.empty(K.q4m_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    K.q4m_pack(torch.from_numpy(w).to(cuda), q, rows, cols)
    x = torch.from_numpy(np.random.default_rng(cols).standard_normal(cols).astype(np.float32)).to(cuda)
    ws = torch.zeros(K.gemv_q4m_workspace_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    want = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4m(q, x, want, rows, cols, workspace=ws)
    y1 = torch.full((rows,), float("nan"), dtype=torch.float32, device=cuda)
    y2 = torch.full((rows,), float("nan"), dtype=torch.float32, device=cuda)
    assert noalloc(q, x, y1, rows, cols) == JINF_OK
    assert noalloc(q, x, y2, rows, cols) == JINF_OK   # counters were left at zero by the first call
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert rel_err(y1.cpu().numpy(), want.cpu().numpy()) < REL
    if rows * cols <= 4096 * 4096:
        assert rel_err(y1.cpu().numpy(), oracle.matvec(w, 2, x.cpu().numpy(), rows, cols)) < REL


def test_noalloc_fp16_input(cuda):
    from jinf import kernels as K
    rows, cols = 6144, 4096
    w = q4_0_rows(rows, cols, seed=7)
    q = torch.empty(K.q4m_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    K.q4m_pack(torch.from_numpy(w).to(cuda), q, rows, cols)
    x16 = np.random.default_rng(3).standard_normal(cols).astype(np.float16)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    assert noalloc(q, torch.from_numpy(x16).to(cuda), y, rows, cols) == JINF_OK
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 2, x16.astype(np.float32), rows, cols)) < REL


def test_noalloc_rejects_oversize_and_bad_arguments(cuda):
    dummy = torch.zeros(64, dtype=torch.uint8, device=cuda)
    xf = torch.zeros(128, dtype=torch.float32, device=cuda)
    y = torch.zeros(16, dtype=torch.float32, device=cuda)
    # 8193 tile pairs of 32 rows: beyond the static scratch (checked before any memory is touched)
    assert noalloc(dummy, xf, y, 8193 * 32, 128) == JINF_ERR_INVALID
    assert noalloc(dummy, xf, y, 16, 100) == JINF_ERR_INVALID   # cols not a multiple of 32
