"""Tensor-parallel decode (q/k/v, gate/up and the vocabulary split by rows, o and down by
columns, a sum over the ranks after each row-split GEMV) on 2 GPUs, one process per GPU, in
both forms: the persistent step (one kernel per token per rank; the partial outputs cross
NVLink into every rank's exchange area) and one kernel per operation (NCCL allreduce). The
gathered logits and the greedy tokens match the CPU oracle. Skipped with fewer than 2 GPUs."""
import os
import queue

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle

pytestmark = pytest.mark.gpu

LOGIT_REL = 1e-2
WORLD = 2


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def _rank_main(rank, world, nccl_id, shape_args, prompt, n_greedy, persistent, kv_pos, out_q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "jetson-inference_b200"))
    try:
        import jinf
        torch.cuda.set_device(rank)
        shape = jinf.LlamaShape(*shape_args)
        syn = jinf.SynthModel(shape, seed=0)
        opts = jinf.b200_options(device=rank, tp_rank=rank, tp_size=world, nccl_id=nccl_id, eos_token=-1,
                                 persistent=persistent)
        eng = jinf.Engine.from_synth(syn, max_context=kv_pos + 64, options=opts)
        kv = None
        if kv_pos:  # the same seeded cache on every rank; the parent gathers the ranks' heads
            eng.fill_kv_random(kv_pos, seed=1)
            kv = eng.kv_read(kv_pos, tp_size=world)
        logits = [eng.logits_host(prompt)]
        toks = [eng.last_argmax()]
        for _ in range(n_greedy):
            logits.append(eng.logits_host([toks[-1]]))
            toks.append(eng.last_argmax())
        persistent = eng.persistent
        eng.close()
        out_q.put((rank, "ok", [l.copy() for l in logits], toks, (persistent, kv)))
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, "error", repr(e), None, None))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("shape_args,kv_pos", [((4, 512, 8, 2, 1408, 4096, 1e4), 0),
                                                ((2, 4096, 32, 8, 14336, 32000, 5e5), 0),
                                                ((2, 4096, 32, 8, 14336, 32000, 5e5), 512)],
                         ids=["tiny", "8b_layers", "8b_layers_pos512"])
@pytest.mark.parametrize("persistent", [True, False], ids=["persistent", "per_op"])
def test_tp2_matches_oracle(shape_args, kv_pos, persistent):
    """kv_pos 512: both sides start from the same 512-position cache (each rank's seeded
    fill, gathered for the oracle), so attention runs at the benchmark's positions."""
    import jinf
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, shape_args[5], size=8)]
    n_greedy = 4
    nccl_id = jinf.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, WORLD, nccl_id, shape_args, prompt, n_greedy, persistent, kv_pos, q))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, status, logits, toks, extra = q.get(timeout=300)
            assert status == "ok", f"rank {rank}: {logits}"
            results[rank] = (logits, toks, extra[0], extra[1])
    except queue.Empty:
        pytest.fail("a tensor-parallel rank did not report within 300 s")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert results[0][2] == persistent and results[1][2] == persistent, "the requested form runs on both ranks"
    # both ranks see the same gathered logits and argmax tokens
    for a, b in zip(results[0][0], results[1][0]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert results[0][1] == results[1][1]
    # against the oracle, token by token
    syn = jinf.SynthModel(jinf.LlamaShape(*shape_args), seed=0)
    orc = oracle.OracleModel(syn, max_ctx=kv_pos + 64, kv_f16=True)
    if kv_pos:
        orc.load_kv_f16(np.concatenate([results[r][3][0] for r in range(WORLD)], axis=1),
                        np.concatenate([results[r][3][1] for r in range(WORLD)], axis=1))
    want = None
    for t in prompt:
        want = orc.forward(t)
    logits, toks = results[0][0], results[0][1]
    for step in range(n_greedy + 1):
        assert rel_err(logits[step], want) < LOGIT_REL, f"step {step}"
        assert toks[step] == oracle.argmax(want), f"step {step}"
        want = orc.forward(toks[step])


def _rank_nvmw_main(rank, world, nccl_id, nvmw, shape_args, prompt, persistent, out_q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "jetson-inference_b200"))
    try:
        import jinf
        from jinf import _lib as L
        torch.cuda.set_device(rank)
        syn = jinf.SynthModel(jinf.LlamaShape(*shape_args), seed=2, weight_type=L.Q4_K, mix_type=L.Q6_K)
        out = []
        for src in ("nvmw", "synth"):
            opts = jinf.b200_options(device=rank, tp_rank=rank, tp_size=world, nccl_id=nccl_id[src], eos_token=-1,
                                     persistent=persistent)
            eng = (jinf.Engine.from_nvmw(nvmw, max_context=64, options=opts) if src == "nvmw"
                   else jinf.Engine.from_synth(syn, max_context=64, options=opts))
            logits = [eng.logits_host(prompt)]
            for _ in range(4):
                logits.append(eng.logits_host([eng.last_argmax()]))
            eng.close()
            out.append([l.copy() for l in logits])
        out_q.put((rank, "ok", out))
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, "error", repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("persistent", [True, False], ids=["persistent", "per_op"])
def test_tp2_from_b200_layout_shards(tmp_path, persistent):
    """Each rank of a 2-GPU engine loads its own pre-packed shard images from a
    jinf_prepare_model_b200_tp file (Q4_K with Q6_K v / down / output) and computes logits
    bit-identical to the same engine built from the reference blocks."""
    import jinf
    from jinf import _lib as L
    shape_args = (2, 1024, 16, 4, 2048, 4096, 1e4)
    syn = jinf.SynthModel(jinf.LlamaShape(*shape_args), seed=2, weight_type=L.Q4_K, mix_type=L.Q6_K)
    gguf, nvmw = str(tmp_path / "m.gguf"), str(tmp_path / "m.nvmw")
    syn.write_gguf(gguf)
    assert L.lib.jinf_prepare_model_b200_tp(gguf.encode(), nvmw.encode(), WORLD) == 0
    prompt = [int(t) for t in np.random.default_rng(1).integers(0, 4096, size=6)]
    ids = {"nvmw": jinf.nccl_unique_id(), "synth": jinf.nccl_unique_id()}
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_nvmw_main, args=(r, WORLD, ids, nvmw, shape_args, prompt, persistent, q))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        for _ in range(WORLD):
            rank, status, out = q.get(timeout=300)
            assert status == "ok", f"rank {rank}: {out}"
            for a, b in zip(out[0], out[1]):
                assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"rank {rank}"
    except queue.Empty:
        pytest.fail("a tensor-parallel rank did not report within 300 s")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()


def _rank_multi_main(rank, world, nccl_id, shape_args, prompts, n_greedy, out_q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "jetson-inference_b200"))
    try:
        import jinf
        torch.cuda.set_device(rank)
        syn = jinf.SynthModel(jinf.LlamaShape(*shape_args), seed=0)
        opts = jinf.b200_options(device=rank, tp_rank=rank, tp_size=world, nccl_id=nccl_id, eos_token=-1,
                                 max_seqs=len(prompts))
        eng = jinf.Engine.from_synth(syn, max_context=64, options=opts)
        seqs = list(range(len(prompts)))
        toks = []
        for t in range(len(prompts[0])):
            toks.append(eng.decode_batch(seqs, [p[t] for p in prompts]))
        for _ in range(n_greedy):
            toks.append(eng.decode_batch(seqs, toks[-1]))
        eng.close()
        out_q.put((rank, "ok", toks))
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, "error", repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_tp2_multi_sequence_greedy_tokens():
    """The multi-sequence step on 2 GPUs (row-split partial outputs summed by NCCL, argmax keys
    max-reduced): three sequences' greedy tokens, identical on both ranks and equal to each
    sequence's own oracle decode."""
    import jinf
    shape_args = (2, 512, 8, 2, 1408, 4096, 1e4)
    rng = np.random.default_rng(7)
    prompts = [[int(t) for t in rng.integers(0, 4096, size=6)] for _ in range(3)]
    n_greedy = 8
    nccl_id = jinf.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_multi_main, args=(r, WORLD, nccl_id, shape_args, prompts, n_greedy, q))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, status, toks = q.get(timeout=300)
            assert status == "ok", f"rank {rank}: {toks}"
            res[rank] = toks
    except queue.Empty:
        pytest.fail("a tensor-parallel rank did not report within 300 s")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[0] == res[1]
    syn = jinf.SynthModel(jinf.LlamaShape(*shape_args), seed=0)
    for i, pr in enumerate(prompts):
        orc = oracle.OracleModel(syn, max_ctx=64, kv_f16=True)
        want = None
        for t in pr:
            want = orc.forward(t)
        steps = len(pr) - 1
        assert res[0][steps][i] == oracle.argmax(want), f"sequence {i} after its prompt"
        for k in range(n_greedy):
            want = orc.forward(res[0][steps + k][i])
            assert res[0][steps + k + 1][i] == oracle.argmax(want), f"sequence {i} step {k}"
        orc.close()
