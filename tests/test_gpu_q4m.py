"""The tensor-core Q4M GEMV (jinf_b200_q4m_* / jinf_b200_gemv_q4m*) on the GPU: the device
repack against the numpy statement of the layout (bit-exact), the GEMV against the CPU
oracle (reference cuda/matmul_kernels.cu:8-43) within 1e-3 relative, for every K split, and
against the numpy statement of its own arithmetic (int8 digit records) within fp32
summation-order noise."""
import numpy as np
import pytest
import torch

import q4m_ref
from oracle import oracle
from test_q4m_layout import q4_0_rows, rel_err

pytestmark = pytest.mark.gpu

REL = 1e-3

SHAPES = [(4096, 4096), (1024, 4096), (6144, 4096), (28672, 4096), (4096, 14336), (4096, 512), (4096, 1792),
          (768, 512), (2816, 512), (512, 1408), (1, 128), (37, 384), (130, 4096), (128256, 4096),
          (512, 704), (40, 96), (4096, 7168)]


def packed(w, rows, cols, cuda):
    from jinf import kernels as K
    q = torch.empty(K.q4m_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    K.q4m_pack(torch.from_numpy(np.ascontiguousarray(w)).to(cuda), q, rows, cols)
    return q


def workspace(rows, cols, cuda):
    from jinf import kernels as K
    return torch.zeros(K.gemv_q4m_workspace_bytes(rows, cols), dtype=torch.uint8, device=cuda)


@pytest.mark.parametrize("rows,cols", [(16, 128), (37, 384), (100, 1408), (4096, 4096), (24, 704), (16, 96)])
def test_q4m_pack_matches_layout(cuda, rows, cols):
    w = q4_0_rows(rows, cols, seed=rows)
    got = packed(w, rows, cols, cuda).cpu().numpy()
    assert np.array_equal(got, q4m_ref.pack(w, rows, cols))


@pytest.mark.parametrize("rows,cols", [(64, 1024), (96, 704), (4096, 4096), (512, 14336)])
def test_gemv_q4m_follows_documented_arithmetic(cuda, rows, cols):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=rows + cols)
    rng = np.random.default_rng(rows)
    x = (rng.standard_normal(cols) * np.repeat(10.0 ** rng.integers(-3, 3, size=cols // 32), 32)).astype(np.float32)
    x[:32] = 0.0                                   # an all-zero block: zero records
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4m(q, torch.from_numpy(x).to(cuda), y, rows, cols, workspace=workspace(rows, cols, cuda), kw=1)
    torch.cuda.synchronize()
    want = q4m_ref.emulate_gemv(q4m_ref.pack(w, rows, cols), x, rows, cols)
    assert rel_err(y.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_q4m_fp32(cuda, rows, cols):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=rows + 3 * cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    q = packed(w, rows, cols, cuda)
    ws = workspace(rows, cols, cuda)
    xd = torch.from_numpy(x).to(cuda)
    y1 = torch.empty(rows, dtype=torch.float32, device=cuda)
    y2 = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4m(q, xd, y1, rows, cols, workspace=ws)
    K.gemv_q4m(q, xd, y2, rows, cols, workspace=ws)  # counters reset themselves; deterministic sums
    torch.cuda.synchronize()
    want = oracle.matvec(w, 2, x, rows, cols)
    assert rel_err(y1.cpu().numpy(), want) < REL
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("rows,cols,kw", [(4096, 4096, 1), (4096, 4096, 2), (4096, 4096, 3), (4096, 4096, 32),
                                          (37, 384, 3), (512, 1408, 11), (130, 4096, 7)])
def test_gemv_q4m_every_k_split(cuda, rows, cols, kw):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=kw)
    x = np.random.default_rng(kw).standard_normal(cols).astype(np.float32)
    q = packed(w, rows, cols, cuda)
    ws = workspace(rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    ref = None
    for _ in range(3):
        K.gemv_q4m(q, torch.from_numpy(x).to(cuda), y, rows, cols, workspace=ws if kw > 1 else None, kw=kw)
        torch.cuda.synchronize()
        if ref is None:
            ref = y.clone()
        assert torch.equal(y, ref)
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 2, x, rows, cols)) < REL


def test_gemv_q4m_rejects_bad_split(cuda):
    import jinf
    from jinf import kernels as K
    q = torch.zeros(K.q4m_bytes(16, 256), dtype=torch.uint8, device=cuda)
    x = torch.zeros(256, dtype=torch.float32, device=cuda)
    y = torch.zeros(16, dtype=torch.float32, device=cuda)
    with pytest.raises(jinf.JinfError):
        K.gemv_q4m(q, x, y, 16, 256, workspace=None, kw=2)   # kw > 1 without a workspace
    ws = workspace(16, 256, cuda)
    with pytest.raises(jinf.JinfError):
        K.gemv_q4m(q, x, y, 16, 256, workspace=ws, kw=3)     # more parts than groups


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (128256, 4096), (4096, 14336)])
def test_gemv_q4m_fp16_input(cuda, rows, cols):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=11)
    x16 = np.random.default_rng(2).standard_normal(cols).astype(np.float16)
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4m(q, torch.from_numpy(x16).to(cuda), y, rows, cols, workspace=workspace(rows, cols, cuda))
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 2, x16.astype(np.float32), rows, cols)) < REL


@pytest.mark.parametrize("xscale", [1e-6, 1.0, 1e5])
def test_gemv_q4m_extreme_values(cuda, xscale):
    """Every nibble value, scales from 1e-7 to 65504, inputs from 1e-6 to 1e5."""
    from jinf import kernels as K
    rows, cols = 64, 1024
    rng = np.random.default_rng(0)
    w = rng.integers(0, 256, size=(rows, cols // 32, 18), dtype=np.uint8)
    d = np.array([1e-7, 6e-5, 1.0, 300.0, -2.5, 65504.0], dtype=np.float16)
    w[..., 0:2] = np.frombuffer(rng.choice(d, size=rows * cols // 32).astype(np.float16).tobytes(),
                                dtype=np.uint8).reshape(rows, cols // 32, 2)
    w = w.reshape(rows, -1)
    x = (rng.standard_normal(cols) * xscale).astype(np.float32)
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4m(q, torch.from_numpy(x).to(cuda), y, rows, cols, workspace=workspace(rows, cols, cuda))
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 2, x, rows, cols)) < REL


@pytest.mark.parametrize("rows,cols", [(6144, 4096), (768, 512)])
def test_gemv_q4m_rmsnorm_prologue(cuda, rows, cols):
    from jinf import kernels as K
    rng = np.random.default_rng(rows)
    w = q4_0_rows(rows, cols, seed=5)
    h = rng.standard_normal(cols).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4m_rmsnorm(q, torch.from_numpy(h).to(cuda), torch.from_numpy(g).to(cuda), 1e-5, y, rows, cols,
                       workspace=workspace(rows, cols, cuda))
    want = oracle.matvec(w, 2, oracle.rmsnorm(h, g, 1e-5), rows, cols)
    assert rel_err(y.cpu().numpy(), want) < REL


# ---------------------------------------------------------------- Q4_K weights

def packed_k(w, rows, cols, cuda):
    from jinf import kernels as K
    q = torch.empty(K.q4m_bytes_qt(rows, cols, 12), dtype=torch.uint8, device=cuda)
    K.q4m_pack_qt(torch.from_numpy(np.ascontiguousarray(w)).to(cuda), 12, q, rows, cols)
    return q


@pytest.mark.parametrize("rows,cols", [(16, 256), (37, 512), (100, 1024), (4096, 4096)])
def test_q4k_pack_matches_layout(cuda, rows, cols):
    from test_q4m_layout import q4_k_rows
    w = q4_k_rows(rows, cols, seed=rows)
    assert np.array_equal(packed_k(w, rows, cols, cuda).cpu().numpy(), q4m_ref.pack_q4k(w, rows, cols))


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 8192), (8192, 1024), (3584, 8192), (8192, 3584),
                                       (16032, 8192), (37, 512), (128, 14336)])
def test_gemv_q4k(cuda, rows, cols):
    from jinf import kernels as K
    from test_q4m_layout import q4_k_rows
    w = q4_k_rows(rows, cols, seed=rows + cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    q = packed_k(w, rows, cols, cuda)
    ws = workspace(rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    y2 = torch.empty(rows, dtype=torch.float32, device=cuda)
    xd = torch.from_numpy(x).to(cuda)
    K.gemv_q4m_qt(q, 12, xd, y, rows, cols, workspace=ws)
    K.gemv_q4m_qt(q, 12, xd, y2, rows, cols, workspace=ws)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 12, x, rows, cols)) < REL
    assert torch.equal(y, y2)
    if rows * cols <= 4096 * 4096:
        want = q4m_ref.emulate_gemv_q4k(q4m_ref.pack_q4k(w, rows, cols), x, rows, cols)
        assert rel_err(y.cpu().numpy(), want) < 1e-5


def test_q4k_rejects_partial_superblocks(cuda):
    from jinf import kernels as K
    assert K.q4m_bytes_qt(16, 384, 12) == 0       # not whole 256-element super-blocks
    assert K.q4m_bytes_qt(16, 384, 2) > 0
    assert K.q4m_bytes_qt(16, 384, 14) == 0       # Q6_K: whole super-blocks too
    assert K.q4m_bytes_qt(16, 96, 8) > 0           # Q8_0: whole 32-element blocks
    assert K.q4m_bytes_qt(16, 256, 1) == 0         # F16: no Q4M form


# ---------------------------------------------------------------- Q6_K and Q8_0 weights

QT_HELPERS = {14: (q4m_ref.random_q6k_rows, q4m_ref.pack_q6k, q4m_ref.emulate_gemv_q6k),
              8: (q4m_ref.random_q80_rows, q4m_ref.pack_q80, q4m_ref.emulate_gemv_q80)}


def packed_qt(w, qt, rows, cols, cuda):
    from jinf import kernels as K
    q = torch.empty(K.q4m_bytes_qt(rows, cols, qt), dtype=torch.uint8, device=cuda)
    K.q4m_pack_qt(torch.from_numpy(np.ascontiguousarray(w)).to(cuda), qt, q, rows, cols)
    return q


@pytest.mark.parametrize("qt,rows,cols", [(14, 16, 256), (14, 37, 512), (14, 100, 1024), (14, 1024, 4096),
                                          (8, 16, 32), (8, 37, 160), (8, 100, 736), (8, 1024, 4096)])
def test_q6k_q80_pack_matches_layout(cuda, qt, rows, cols):
    gen, pack, _ = QT_HELPERS[qt]
    w = gen(rows, cols, seed=rows + qt)
    assert np.array_equal(packed_qt(w, qt, rows, cols, cuda).cpu().numpy(), pack(w, rows, cols))


@pytest.mark.parametrize("qt,rows,cols", [(14, 4096, 4096), (14, 1024, 4096), (14, 4096, 14336), (14, 128256, 4096),
                                          (14, 37, 512), (14, 8192, 1024), (14, 8192, 28672),
                                          (8, 4096, 4096), (8, 1024, 4096), (8, 4096, 14336), (8, 128256, 4096),
                                          (8, 37, 160), (8, 40, 96), (8, 8192, 28672)])
def test_gemv_q6k_q80(cuda, qt, rows, cols):
    from jinf import kernels as K
    gen, pack, emulate = QT_HELPERS[qt]
    w = gen(rows, cols, seed=rows + cols + qt)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    q = packed_qt(w, qt, rows, cols, cuda)
    ws = workspace(rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    y2 = torch.empty(rows, dtype=torch.float32, device=cuda)
    xd = torch.from_numpy(x).to(cuda)
    K.gemv_q4m_qt(q, qt, xd, y, rows, cols, workspace=ws)
    K.gemv_q4m_qt(q, qt, xd, y2, rows, cols, workspace=ws)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, qt, x, rows, cols)) < REL
    assert torch.equal(y, y2)
    if rows * cols <= 1024 * 4096:
        assert rel_err(y.cpu().numpy(), emulate(pack(w, rows, cols), x, rows, cols)) < 1e-5


@pytest.mark.parametrize("qt", [14, 8])
@pytest.mark.parametrize("kw", [1, 2, 3, 7, 32])
def test_gemv_q6k_q80_every_k_split(cuda, qt, kw):
    from jinf import kernels as K
    rows, cols = 2048, 4096
    gen = QT_HELPERS[qt][0]
    w = gen(rows, cols, seed=kw + qt)
    x = np.random.default_rng(kw).standard_normal(cols).astype(np.float32)
    q = packed_qt(w, qt, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4m_qt(q, qt, torch.from_numpy(x).to(cuda), y, rows, cols, workspace=workspace(rows, cols, cuda), kw=kw)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, qt, x, rows, cols)) < REL


# ---------------------------------------------------------------- batched GEMV (C2 at batch 4 / 8)

@pytest.mark.parametrize("rows,cols,batch", [(4096, 4096, 4), (4096, 4096, 8), (1024, 4096, 8), (14336, 4096, 4),
                                             (4096, 14336, 8), (37, 384, 3), (128256, 4096, 8), (512, 704, 5),
                                             (4096, 4096, 1)])
def test_gemv_q4m_batch(cuda, rows, cols, batch):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=rows + cols + batch)
    x = np.random.default_rng(batch).standard_normal((batch, cols)).astype(np.float16)
    q = packed(w, rows, cols, cuda)
    ws = torch.zeros(K.gemv_q4m_batch_workspace_bytes(rows, cols, batch), dtype=torch.uint8, device=cuda)
    xd = torch.from_numpy(x).to(cuda)
    y = torch.empty((batch, rows), dtype=torch.float32, device=cuda)
    y2 = torch.empty_like(y)
    K.gemv_q4m_batch(q, xd, y, rows, cols, batch, workspace=ws)
    K.gemv_q4m_batch(q, xd, y2, rows, cols, batch, workspace=ws)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for b in range(batch):
        assert rel_err(got[b], oracle.matvec(w, 2, x[b].astype(np.float32), rows, cols)) < REL, f"vector {b}"
    assert torch.equal(y, y2)
    if rows * cols <= 4096 * 4096:
        for b in range(min(batch, 2)):
            want = q4m_ref.emulate_gemv(q4m_ref.pack(w, rows, cols), x[b].astype(np.float32), rows, cols)
            assert rel_err(got[b], want) < 1e-5


# ---------------------------------------------------------------- multi-vector GEMV, every format

def _typed_rows(qt, rows, cols, seed):
    from test_q4m_layout import q4_k_rows
    if qt == 2:
        return q4_0_rows(rows, cols, seed=seed)
    if qt == 12:
        return q4_k_rows(rows, cols, seed=seed)
    return QT_HELPERS[qt][0](rows, cols, seed=seed)


@pytest.mark.parametrize("qt", [2, 12, 14, 8])
@pytest.mark.parametrize("rows,cols,batch", [(4096, 4096, 8), (1024, 8192, 3), (3584, 8192, 8), (8192, 3584, 5),
                                             (160, 1024, 1), (128256, 4096, 8)])
def test_gemv_batch_every_format(cuda, qt, rows, cols, batch):
    """Y[b] = W x[b] through the multi-vector kernel (the engine's multi-sequence GEMV) against
    the oracle's matvec of each vector, for Q4_0, Q4_K, Q6_K and Q8_0 images; deterministic."""
    from jinf import kernels as K
    w = _typed_rows(qt, rows, cols, seed=rows + cols + qt)
    q = packed_qt(w, qt, rows, cols, cuda) if qt != 12 else packed_k(w, rows, cols, cuda)
    x = np.random.default_rng(batch + qt).standard_normal((batch, cols)).astype(np.float32)
    ws = torch.zeros(K.gemv_q4m_batch_workspace_bytes_qt(rows, cols, batch, qt), dtype=torch.uint8, device=cuda)
    xd = torch.from_numpy(x).to(cuda)
    y = torch.empty((batch, rows), dtype=torch.float32, device=cuda)
    y2 = torch.empty_like(y)
    K.gemv_q4m_batch_qt(q, qt, xd, y, rows, cols, batch, workspace=ws)
    K.gemv_q4m_batch_qt(q, qt, xd, y2, rows, cols, batch, workspace=ws)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for b in range(batch):
        assert rel_err(got[b], oracle.matvec(w, qt, x[b], rows, cols)) < REL, f"vector {b}"
    assert torch.equal(y, y2)


@pytest.mark.parametrize("qt", [2, 12, 14, 8])
@pytest.mark.parametrize("kw", [1, 2, 5, 16, -1, -2, -3, -16])
def test_gemv_batch_every_k_split(cuda, qt, kw):
    """Every forced K split gives the same vectors (to the oracle bar) and matches kw = 1 to
    fp32 summation order; kw < 0: -kw parts with a CTA's warps splitting each tile pair.
    (2048 columns: at 8 vectors the records of all 16 groups fit in shared memory, so one
    part is a valid split for every format.)"""
    from jinf import kernels as K
    rows, cols, batch = 1024, 2048, 8
    w = _typed_rows(qt, rows, cols, seed=7 * abs(kw) + qt)
    q = packed_qt(w, qt, rows, cols, cuda) if qt != 12 else packed_k(w, rows, cols, cuda)
    x = np.random.default_rng(abs(kw)).standard_normal((batch, cols)).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda)
    ws = torch.zeros(K.gemv_q4m_batch_workspace_bytes_qt(rows, cols, batch, qt), dtype=torch.uint8, device=cuda)
    y = torch.empty((batch, rows), dtype=torch.float32, device=cuda)
    K.gemv_q4m_batch_qt(q, qt, xd, y, rows, cols, batch, workspace=ws, kw=kw)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for b in range(batch):
        assert rel_err(got[b], oracle.matvec(w, qt, x[b], rows, cols)) < REL, f"vector {b}"
