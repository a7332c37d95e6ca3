"""The engine's B200 building blocks (jinf_b200_*) on the GPU against the CPU oracle:
Q4T repack + fused GEMV, the RMSNorm-prologue GEMV and the fp16-KV split-K attention."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

REL = 1e-3


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def q4_0_rows(rows, cols, seed, std=0.02):
    import jinf
    x = (np.random.default_rng(seed).standard_normal(rows * cols) * std).astype(np.float32)
    out = np.empty(rows * cols // 32 * 18, dtype=np.uint8)
    jinf.lib.jinf_quantize_q4_0(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), rows * cols)
    return out.reshape(rows, -1)


def packed(w, rows, cols, cuda):
    from jinf import kernels as K
    n = K.q4t_bytes(rows, cols)
    assert n > 0
    q = torch.empty(n, dtype=torch.uint8, device=cuda)
    K.q4t_pack(torch.from_numpy(w).to(cuda), q, rows, cols)
    return q


# 8B projection shapes (out x in), the tiny config's, tensor-parallel shards, ragged rows
GEMV_SHAPES = [(4096, 4096), (1024, 4096), (6144, 4096), (28672, 4096), (4096, 14336), (4096, 512), (4096, 1792),
               (768, 512), (2816, 512), (512, 1408), (4096, 512), (1, 128), (37, 384), (130, 4096)]


@pytest.mark.parametrize("rows,cols", GEMV_SHAPES)
def test_gemv_q4t_fp32(cuda, rows, cols):
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=rows + 3 * cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4t(q, torch.from_numpy(x).to(cuda), y, rows, cols)
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 2, x, rows, cols)) < REL


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (128256, 4096), (4096, 14336)])
def test_gemv_q4t_fp16_input(cuda, rows, cols):
    """C2 microbench convention: x fp16 N(0,1), the oracle takes the same x upcast to fp32."""
    from jinf import kernels as K
    w = q4_0_rows(rows, cols, seed=11)
    x16 = np.random.default_rng(2).standard_normal(cols).astype(np.float16)
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4t(q, torch.from_numpy(x16).to(cuda), y, rows, cols)
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 2, x16.astype(np.float32), rows, cols)) < REL


def test_gemv_q4t_extreme_values(cuda):
    """Every nibble value and large/small scales: the magic-exponent decode is exact."""
    from jinf import kernels as K
    rows, cols = 64, 1024
    rng = np.random.default_rng(0)
    w = rng.integers(0, 256, size=(rows, cols // 32, 18), dtype=np.uint8)
    d = np.array([1e-7, 6e-5, 1.0, 300.0, -2.5, 65504.0], dtype=np.float16)
    w[..., 0:2] = np.frombuffer(rng.choice(d, size=rows * cols // 32).astype(np.float16).tobytes(),
                                dtype=np.uint8).reshape(rows, cols // 32, 2)
    w = w.reshape(rows, -1)
    x = rng.standard_normal(cols).astype(np.float32)
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4t(q, torch.from_numpy(x).to(cuda), y, rows, cols)
    assert rel_err(y.cpu().numpy(), oracle.matvec(w, 2, x, rows, cols)) < REL


def test_q4t_pack_is_lossless(cuda):
    """Every nibble byte and scale of the AoS matrix appears exactly once in the Q4T image."""
    from jinf import kernels as K
    rows, cols = 100, 1408
    w = q4_0_rows(rows, cols, seed=4)
    q = packed(w, rows, cols, cuda).cpu().numpy()
    nib = np.sort(w.reshape(-1, 18)[:, 2:].reshape(-1))
    sc = np.sort(w.reshape(-1, 18)[:, :2].copy().view(np.uint16).reshape(-1))
    total = K.q4t_bytes(rows, cols)
    chunks = q.reshape(-1, 2304)
    qn = chunks[:, :2048].reshape(-1)
    qs = chunks[:, 2048:].copy().view(np.uint16).reshape(-1)
    # padding rows are zero: drop as many zeros as padding contributes
    pad_blocks = qn.size // 16 - rows * cols // 32
    assert total == chunks.size
    assert np.array_equal(np.sort(qn)[pad_blocks * 16:], nib)
    assert np.array_equal(np.sort(qs)[pad_blocks:], sc)


@pytest.mark.parametrize("rows,cols", [(6144, 4096), (768, 512)])
def test_gemv_q4t_rmsnorm_prologue(cuda, rows, cols):
    from jinf import kernels as K
    rng = np.random.default_rng(rows)
    w = q4_0_rows(rows, cols, seed=5)
    h = rng.standard_normal(cols).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    q = packed(w, rows, cols, cuda)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_q4t_rmsnorm(q, torch.from_numpy(h).to(cuda), torch.from_numpy(g).to(cuda), 1e-5, y, rows, cols)
    want = oracle.matvec(w, 2, oracle.rmsnorm(h, g, 1e-5), rows, cols)
    assert rel_err(y.cpu().numpy(), want) < REL


@pytest.mark.parametrize("hd,nh,nkv,n_pos,max_ctx", [(64, 8, 2, 1, 128), (64, 8, 2, 100, 128), (128, 32, 8, 769, 800),
                                                     (128, 64, 8, 8192, 8192), (128, 4, 1, 4097, 8192)])
def test_attention_f16(cuda, hd, nh, nkv, n_pos, max_ctx):
    from jinf import kernels as K
    rng = np.random.default_rng(n_pos)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    kc = rng.standard_normal((nkv, max_ctx, hd)).astype(np.float16)
    vc = rng.standard_normal((nkv, max_ctx, hd)).astype(np.float16)
    ws = torch.zeros(K.attention_workspace_bytes(nkv, hd, max_ctx), dtype=torch.uint8, device=cuda)
    out = torch.empty(nh * hd, dtype=torch.float32, device=cuda)
    for _ in range(2):  # the self-resetting split counters must survive back-to-back calls
        K.attention_f16(out, torch.from_numpy(q).to(cuda), torch.from_numpy(kc).to(cuda),
                        torch.from_numpy(vc).to(cuda), hd, nh, nkv, n_pos, max_ctx, ws)
        torch.cuda.synchronize()
    # oracle in the reference layout [ctx][nkv*hd] with the same fp16 values
    kr = kc.astype(np.float32).transpose(1, 0, 2).reshape(max_ctx, nkv * hd)
    vr = vc.astype(np.float32).transpose(1, 0, 2).reshape(max_ctx, nkv * hd)
    assert rel_err(out.cpu().numpy(), oracle.attention(q, kr, vr, hd, nh, nkv, n_pos)) < REL


@pytest.mark.parametrize("name,row0,n", [("blk.0.attn_q.weight", 0, 512), ("blk.3.ffn_down.weight", 100, 300),
                                         ("token_embd.weight", 4000, 96), ("output.weight", 7, 1),
                                         ("blk.1.ffn_norm.weight", 0, 1)])
def test_device_generator_bit_identical_to_host(cuda, name, row0, n):
    """The GPU weight generator reproduces the host generator's bytes exactly."""
    import jinf
    syn = jinf.SynthModel(jinf.TINY, seed=0)
    host = syn.read_rows(name, row0, n)
    out = torch.empty(host.nbytes, dtype=torch.uint8, device=cuda)
    syn.read_rows_device(name, out, row0, n)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), host.reshape(-1).view(np.uint8))
