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


# ---------------------------------------------------------------- the engine's batched prefill

def rel_logits(got, want):
    return float(np.max(np.abs(np.asarray(got, np.float64) - want)) / max(np.max(np.abs(want)), 1e-30))


def top_gap(v):
    t = np.sort(v)[-2:]
    return float(t[1] - t[0])


def _prefill_vs_oracle(syn, prompt, n_greedy, max_ctx):
    import jinf
    eng = jinf.Engine.from_synth(syn, max_context=max_ctx, options=jinf.b200_options(eos_token=-1, prefill=True))
    orc = oracle.OracleModel(syn, max_ctx=max_ctx, kv_f16=True)
    want = None
    for t in prompt:
        want = orc.forward(t)
    got = eng.logits_host(prompt)
    assert eng.n_past == len(prompt)
    worst, gap = rel_logits(got, want), top_gap(want)
    assert worst < 1e-2
    for step in range(n_greedy):
        tok = oracle.argmax(want)
        assert eng.last_argmax() == tok, f"step {step}"
        want = orc.forward(tok)
        got = eng.logits_host([tok])
        e = rel_logits(got, want)
        assert e < 1e-2, f"step {step}: {e:.3g}"
        worst, gap = max(worst, e), min(gap, top_gap(want))
    orc.close()
    eng.close()
    return worst, gap


def test_engine_prefill_tiny_logits_and_32_greedy_tokens(cuda):
    """C1 tiny model: the 16-token prompt's first 15 tokens through the batched prefill (tensor
    cores, causal attention over all of them at once), the last as a decode step; the logits
    and the following 32 greedy tokens against the oracle's token-by-token decode."""
    import jinf
    syn = jinf.SynthModel(jinf.TINY, seed=0)
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, 4096, size=16)]
    worst, gap = _prefill_vs_oracle(syn, prompt, 32, 128)
    print(f"tiny prefill: max logits rel err {worst:.3g}, min top-1/top-2 gap {gap:.3g}")


def test_engine_prefill_8b_layer_two_chunks(cuda):
    """One Llama-3-8B-shaped layer (d 4096, 32/8 heads of 128, ff 14336; vocabulary 32000) with
    a 530-token prompt: prefill chunks of 512 and 17 tokens (the second chunk's attention reads
    the first chunk's cache rows), then 8 greedy steps, against the oracle."""
    import jinf
    shape = jinf.LlamaShape(1, 4096, 32, 8, 14336, 32000, 5e5)
    syn = jinf.SynthModel(shape, seed=6)
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, 32000, size=530)]
    worst, gap = _prefill_vs_oracle(syn, prompt, 8, 560)
    print(f"8B layer prefill (530 tokens): max logits rel err {worst:.3g}, min top-1/top-2 gap {gap:.3g}")


def test_engine_prefill_matches_token_by_token(cuda):
    """The batched prefill and the token-by-token prompt (prefill off) agree to the logits bar,
    and the KV rows they leave in the cache agree to fp16 rounding."""
    import jinf
    shape = jinf.LlamaShape(2, 4096, 32, 8, 14336, 32000, 5e5)
    syn = jinf.SynthModel(shape, seed=8)
    prompt = [int(t) for t in np.random.default_rng(8).integers(0, 32000, size=64)]
    a = jinf.Engine.from_synth(syn, max_context=80, options=jinf.b200_options(eos_token=-1, prefill=True))
    b = jinf.Engine.from_synth(syn, max_context=80, options=jinf.b200_options(eos_token=-1, prefill=False))
    la, lb = a.logits_host(prompt), b.logits_host(prompt)
    assert rel_logits(la, lb) < 1e-2
    assert a.last_argmax() == b.last_argmax()
    ka, va = a.kv_read(len(prompt))
    kb, vb = b.kv_read(len(prompt))
    for x, y in ((ka, kb), (va, vb)):
        x, y = x.astype(np.float32), y.astype(np.float32)
        assert float(np.max(np.abs(x - y)) / np.max(np.abs(y))) < 1e-2
    a.close()
    b.close()
