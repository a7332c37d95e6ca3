"""The engine's fp16-KV split-K decode attention (jinf_b200_attention_f16) and the device
weight generator on the GPU, against the CPU oracle and the host generator."""
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


@pytest.mark.parametrize("name,row0,n", [("blk.0.attn_q.weight", 0, 512), ("blk.3.ffn_down.weight", 100, 300),
                                         ("output.weight", 7, 1)])
def test_device_q4k_generator_bit_identical_to_host(cuda, name, row0, n):
    """Q4_K models: the GPU generator's quantiser reproduces the host quantiser's bytes."""
    import jinf
    from jinf import _lib as L
    syn = jinf.SynthModel(jinf.LlamaShape(4, 512, 8, 2, 1536, 4096, 10000.0, 1e-5), seed=0, weight_type=L.Q4_K)
    host = syn.read_rows(name, row0, n)
    out = torch.empty(host.nbytes, dtype=torch.uint8, device=cuda)
    syn.read_rows_device(name, out, row0, n)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), host.reshape(-1).view(np.uint8))
