"""Reference kernel C-ABI (jinf_cuda_*) on the GPU against the CPU oracle.

Tolerances: dequantization bit-exact; every fp kernel within
1e-3 relative error, measured as max|got - want| / max|want| over the output vector.
"""
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


def same_bits(got, want):
    """Bit equality of fp32 arrays; NaN payloads are not compared (x86 and the GPU produce
    different NaN bit patterns for the golden's NaN/Inf scales), NaN positions are."""
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    gn, wn = np.isnan(got), np.isnan(want)
    return bool(np.array_equal(gn, wn) and np.array_equal(got[~gn].view(np.uint32), want[~wn].view(np.uint32)))


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def quant_rows(rows, cols, qtype, seed):
    """Seeded realistic blocks: normal weights quantized by the library's own quantizers."""
    import ctypes as C
    import jinf
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    be, bb = oracle.BLOCK[qtype]
    out = np.empty(rows * cols // be * bb, dtype=np.uint8)
    fn = jinf.lib.jinf_quantize_q4_0 if qtype == jinf.Q4_0 else jinf.lib.jinf_quantize_q4_K
    fn(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), rows * cols)
    return out.reshape(rows, -1)


@pytest.mark.parametrize("kind,qt,per", [("q4_0", 2, 32), ("q8_0", 8, 32), ("q4_K", 12, 256)])
def test_dequantize_bit_exact_golden(cuda, golden, kind, qt, per):
    from jinf import kernels as K
    b = golden[f"{kind}_blocks"]
    want = golden[f"{kind}_out"]
    out = torch.empty(want.size, dtype=torch.float32, device=cuda)
    K.dequantize(dev(b, cuda), out, b.shape[0], qt)
    assert same_bits(out.cpu().numpy(), want)


def test_dequantize_q6k_matches_oracle_bits(cuda):
    from jinf import kernels as K
    rng = np.random.default_rng(5)
    b = rng.integers(0, 256, size=(33, 210), dtype=np.uint8)
    b[:, 208:210] = np.frombuffer((rng.standard_normal(33) * 0.01).astype(np.float16).tobytes(),
                                  dtype=np.uint8).reshape(33, 2)
    out = torch.empty(33 * 256, dtype=torch.float32, device=cuda)
    K.dequantize(dev(b, cuda), out, 33, 14)
    assert same_bits(out.cpu().numpy(), oracle.dequant(b, 14))


@pytest.mark.parametrize("offset_bytes", [0, 4, 2])
def test_dequantize_unaligned_output(cuda, golden, offset_bytes):
    """The reference ABI accepts any float pointer; misaligned destinations must work."""
    from jinf import kernels as K
    b = golden["q4_0_blocks"][:37]
    want = golden["q4_0_out"][: 37 * 32]
    if offset_bytes % 4:
        pytest.skip("float outputs are at least 4-byte aligned")
    buf = torch.zeros(37 * 32 + 8, dtype=torch.float32, device=cuda)
    view = buf[offset_bytes // 4: offset_bytes // 4 + 37 * 32]
    K.dequantize(dev(b, cuda), view, 37, 2)
    assert same_bits(view.cpu().numpy(), want)


SHAPES = [(512, 512), (128, 512), (1408, 512), (512, 1408), (4096, 512), (1024, 4096), (4096, 14336), (33, 96)]


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("qt", [2, 12])
def test_dequant_matvec(cuda, rows, cols, qt):
    from jinf import kernels as K
    if qt == 12 and cols % 256:
        pytest.skip("Q4_K needs cols % 256 == 0")
    w = quant_rows(rows, cols, qt, seed=rows * 7 + cols)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.dequant_matvec(dev(w, cuda), dev(x, cuda), y, rows, cols, qt)
    want = oracle.matvec(w, qt, x, rows, cols)
    assert rel_err(y.cpu().numpy(), want) < REL


def test_dequant_matvec_q8_0_and_unaligned_input(cuda):
    from jinf import kernels as K
    rng = np.random.default_rng(9)
    rows, cols = 77, 320
    b = rng.integers(0, 256, size=(rows, cols // 32, 34), dtype=np.uint8)
    b[..., 0:2] = np.frombuffer((rng.standard_normal(rows * cols // 32) * 0.01).astype(np.float16).tobytes(),
                                dtype=np.uint8).reshape(rows, cols // 32, 2)
    x = rng.standard_normal(cols + 1).astype(np.float32)
    xd = dev(x, cuda)[1:]  # 4-byte aligned, not 16-byte aligned
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.dequant_matvec(dev(b, cuda), xd, y, rows, cols, 8)
    want = oracle.matvec(b.reshape(rows, -1), 8, x[1:], rows, cols)
    assert rel_err(y.cpu().numpy(), want) < REL


def test_dequant_matvec_unsupported_qtype_reports(cuda):
    import jinf
    from jinf import kernels as K
    w = torch.zeros(64, dtype=torch.uint8, device=cuda)
    x = torch.zeros(32, dtype=torch.float32, device=cuda)
    y = torch.zeros(1, dtype=torch.float32, device=cuda)
    with pytest.raises(jinf.JinfError):
        K.dequant_matvec(w, x, y, 1, 32, 3)


@pytest.mark.parametrize("n", [1, 31, 512, 4096, 8192])
@pytest.mark.parametrize("wtype", [0, 1])
def test_rmsnorm(cuda, n, wtype):
    from jinf import kernels as K
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    wd = dev(w.astype(np.float16) if wtype == 1 else w, cuda)
    K.rmsnorm(out, dev(x, cuda), wd, n, 1e-5, wtype)
    wref = w.astype(np.float16).astype(np.float32) if wtype == 1 else w
    assert rel_err(out.cpu().numpy(), oracle.rmsnorm(x, wref, 1e-5)) < REL


def test_rmsnorm_in_place(cuda):
    from jinf import kernels as K
    x = np.random.default_rng(3).standard_normal(4096).astype(np.float32)
    w = np.ones(4096, dtype=np.float32)
    xd = dev(x, cuda)
    K.rmsnorm(xd, xd, dev(w, cuda), 4096, 1e-5)
    assert rel_err(xd.cpu().numpy(), oracle.rmsnorm(x, w, 1e-5)) < REL


@pytest.mark.parametrize("hd,nh,nkv,pos,base", [(64, 8, 2, 0, 1e4), (64, 8, 2, 127, 1e4), (128, 32, 8, 767, 5e5),
                                                (128, 64, 8, 8191, 5e5)])
def test_rope(cuda, hd, nh, nkv, pos, base):
    from jinf import kernels as K
    rng = np.random.default_rng(pos)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    qd, kd = dev(q, cuda), dev(k, cuda)
    K.rope(qd, kd, hd, nh, nkv, pos, base)
    qw, kw = oracle.rope(q, k, hd, nh, nkv, pos, base)
    assert rel_err(qd.cpu().numpy(), qw) < REL and rel_err(kd.cpu().numpy(), kw) < REL


@pytest.mark.parametrize("n", [1, 1408, 14336, 28672])
def test_silu_mul(cuda, n):
    from jinf import kernels as K
    rng = np.random.default_rng(n)
    g = (3 * rng.standard_normal(n)).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    K.silu_mul(out, dev(g, cuda), dev(u, cuda), n)
    assert rel_err(out.cpu().numpy(), oracle.silu_mul(g, u)) < REL


@pytest.mark.parametrize("n", [1, 100, 4096, 128256])
def test_softmax(cuda, n):
    from jinf import kernels as K
    x = (5 * np.random.default_rng(n).standard_normal(n)).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    K.softmax(out, dev(x, cuda), n)
    assert rel_err(out.cpu().numpy(), oracle.softmax(x)) < REL


def test_residual_add(cuda):
    from jinf import kernels as K
    a = np.random.default_rng(1).standard_normal(4097).astype(np.float32)
    b = np.random.default_rng(2).standard_normal(4097).astype(np.float32)
    ad = dev(a, cuda)
    K.residual_add(ad, dev(b, cuda), 4097)
    assert np.array_equal(ad.cpu().numpy(), a + b)


@pytest.mark.parametrize("hd,nh,nkv,n_past,max_ctx", [(64, 8, 2, 1, 128), (64, 8, 2, 17, 128), (64, 8, 2, 128, 128),
                                                      (128, 32, 8, 768, 800), (128, 64, 8, 300, 512),
                                                      (128, 8, 8, 33, 64), (96, 4, 1, 50, 64)])
def test_attention_f32_reference_layout(cuda, hd, nh, nkv, n_past, max_ctx):
    from jinf import kernels as K
    rng = np.random.default_rng(n_past + nh)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    kc = rng.standard_normal((max_ctx, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((max_ctx, nkv * hd)).astype(np.float32)
    out = torch.empty(nh * hd, dtype=torch.float32, device=cuda)
    K.attention(out, dev(q, cuda), dev(kc, cuda), dev(vc, cuda), hd, nh, nkv, n_past, max_ctx)
    assert rel_err(out.cpu().numpy(), oracle.attention(q, kc, vc, hd, nh, nkv, n_past)) < REL


def test_attention_long_context_no_smem_limit(cuda):
    """The reference kept n_past scores in shared memory (~12k positions); split-K has no limit."""
    from jinf import kernels as K
    hd, nh, nkv, n = 128, 8, 1, 20000
    rng = np.random.default_rng(11)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    kc = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    out = torch.empty(nh * hd, dtype=torch.float32, device=cuda)
    K.attention(out, dev(q, cuda), dev(kc, cuda), dev(vc, cuda), hd, nh, nkv, n, n)
    assert rel_err(out.cpu().numpy(), oracle.attention(q, kc, vc, hd, nh, nkv, n)) < REL


def make_bundles(hidden, n_ff, qt, seed, extra=None):
    """Reference bundle layout: [gate row][up row][down column f32], padded to 4 KB (or, with
    `extra`, to the raw size plus `extra` bytes, which misaligns every other bundle)."""
    rng = np.random.default_rng(seed)
    gate = quant_rows(n_ff, hidden, qt, seed)
    up = quant_rows(n_ff, hidden, qt, seed + 1)
    down = (rng.standard_normal((n_ff, hidden)) * 0.02).astype(np.float32)  # column i of down = row i here
    rb = gate.shape[1]
    raw = 2 * rb + 4 * hidden
    bsz = (raw + 4095) // 4096 * 4096 if extra is None else raw + extra
    buf = np.zeros((n_ff, bsz), dtype=np.uint8)
    buf[:, :rb] = gate
    buf[:, rb:2 * rb] = up
    buf[:, 2 * rb:2 * rb + 4 * hidden] = down.view(np.uint8).reshape(n_ff, -1)
    return buf, bsz


@pytest.mark.parametrize("qt", [2, 12])
@pytest.mark.parametrize("n_act", [0, 1, 97, 215])
def test_sparse_ffn(cuda, qt, n_act):
    from jinf import kernels as K
    hidden, n_ff = 512, 1408
    buf, bsz = make_bundles(hidden, n_ff, qt, seed=qt)
    rng = np.random.default_rng(n_act)
    act = np.sort(rng.choice(n_ff, size=n_act, replace=False)).astype(np.int32)
    offs = (act * bsz).astype(np.int32)
    x = rng.standard_normal(hidden).astype(np.float32)
    out = torch.full((hidden,), 5.0, dtype=torch.float32, device=cuda)
    gu = torch.empty(max(1, n_act), dtype=torch.float32, device=cuda)
    K.sparse_ffn(dev(buf, cuda), dev(x, cuda), out, dev(offs if n_act else np.zeros(1, np.int32), cuda), n_act,
                 hidden, bsz, qt, gu)
    want, want_gu = oracle.sparse_ffn(buf, x, offs, n_act, hidden, qt)
    if n_act == 0:
        assert np.all(out.cpu().numpy() == 0.0)
    else:
        assert rel_err(gu.cpu().numpy()[:n_act], want_gu) < REL
        assert rel_err(out.cpu().numpy(), want) < REL


@pytest.mark.parametrize("hidden,n_act,extra,alias", [
    (4096, 2150, None, False),   # the 8B shape at 15% of 14336 (fewer bundles here)
    (4096, 333, 4, True),        # every other gate row 4 bytes off 8-byte alignment; out aliases x
    (8192, 300, 0, False),       # two 128-block rounds per lane
    (480, 57, 4, True),          # hidden not a multiple of 128: the per-block path
])
def test_sparse_ffn_shapes(cuda, hidden, n_act, extra, alias):
    """Vectorised Q4_0 gate/up and down paths, their alignment fall-backs and an output that
    aliases the input (the reference engine passes the same buffer, src/engine.cpp:404-408)."""
    from jinf import kernels as K
    n_ff = max(n_act + 7, 400)
    buf, bsz = make_bundles(hidden, n_ff, 2, seed=hidden + n_act, extra=extra)
    rng = np.random.default_rng(n_act)
    act = np.sort(rng.choice(n_ff, size=n_act, replace=False)).astype(np.int32)
    offs = (act.astype(np.int64) * bsz).astype(np.int32)
    x = rng.standard_normal(hidden).astype(np.float32)
    want, want_gu = oracle.sparse_ffn(buf, x, offs, n_act, hidden, 2)
    xd = dev(x, cuda)
    out = xd if alias else torch.full((hidden,), 5.0, dtype=torch.float32, device=cuda)
    gu = torch.empty(n_act, dtype=torch.float32, device=cuda)
    K.sparse_ffn(dev(buf, cuda), xd, out, dev(offs, cuda), n_act, hidden, bsz, 2, gu)
    torch.cuda.synchronize()
    assert rel_err(gu.cpu().numpy(), want_gu) < REL
    assert rel_err(out.cpu().numpy(), want) < REL
