"""Regenerates tests/golden/ref_engine_c1.npz from the reference's OWN engine and CUDA
kernels, run on a GPU: oracle/_ref/ref_engine (built unmodified from the reference tree by
oracle/Makefile, with a pread stand-in for its NVMe reader) and oracle/_ref/prepare_model
(the reference's GGUF -> NVMW tool). Needs a CUDA device and those two prebuilt files; the
reference tree itself is not read.

    python tests/golden/make_ref_engine_golden.py [out.npz] [gemv.json]    (repository root)

What it records:
  * C1 tiny decode: the synthetic tiny model (seed 0, Q4_0) written as GGUF, converted by
    the reference tool with every layer resident, then the reference's jinf_engine_forward
    one token at a time over the 16-token prompt and 32 greedy steps (fp32 KV cache, as the
    reference keeps it). Kept: every step's argmax token and the full logits of the steps
    in ref_cases.C1_KEEP.
  * per-kernel outputs of jinf_cuda_dequant_matvec (Q4_0, Q4_K, Q6_K), jinf_cuda_rmsnorm,
    jinf_cuda_rope, jinf_cuda_attention and jinf_cuda_silu_mul on the cases of
    ref_cases.py (inputs rebuilt from their seeds by the tests).
  * optionally (second argument) the reference kernel's dequant-matvec timing on the
    Llama-3-8B projection shapes, as JSON.
"""
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import ref_cases as RC  # noqa: E402
from oracle import oracle  # noqa: E402

REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "ref_engine")
REF_PREPARE = os.path.join(ROOT, "oracle", "_ref", "prepare_model")


def sources():
    cache = {}

    def get(name):
        if name not in cache:
            shp, wt, mt = RC.shapes()[name]
            cache[name] = oracle.SynthSource(shp, seed=0, weight_type=wt, mix_type=mt)
        return cache[name]
    return get


def decode(d: str) -> dict:
    shp, _, _ = RC.shapes()["tiny"]
    gguf, nvmw, out = (os.path.join(d, n) for n in ("tiny.gguf", "tiny.nvmw", "decode.bin"))
    oracle.SynthSource(shp, seed=0).write_gguf(gguf)
    subprocess.run([REF_PREPARE, "--input", gguf, "--output", nvmw, "--gpu-budget", "4500"], check=True,
                   capture_output=True)
    subprocess.run([REF_ENGINE, "decode", nvmw, out, str(RC.C1_CTX), str(RC.C1_GEN)] + [str(t) for t in RC.C1_PROMPT],
                   check=True)
    raw = open(out, "rb").read()
    n_prompt, n_gen, V = struct.unpack_from("<3i", raw, 0)
    n = n_prompt + n_gen
    toks = np.frombuffer(raw, dtype=np.int32, count=n, offset=12)
    logits = np.frombuffer(raw, dtype=np.float32, count=n * V, offset=12 + 4 * n).reshape(n, V)
    return {"c1_tokens": toks.copy(), "c1_keep": np.array(RC.C1_KEEP, dtype=np.int32),
            "c1_logits": logits[RC.C1_KEEP].copy()}


def kernels(d: str) -> dict:
    src = sources()
    fin, fout = os.path.join(d, "cases.bin"), os.path.join(d, "kout.bin")
    sizes, names = [], []
    with open(fin, "wb") as f:
        for case in RC.MATVEC:
            rows, cols, qt, w, x = RC.matvec_inputs(src, case)
            f.write(struct.pack("<5i", 1, rows, cols, qt, w.nbytes) + w.tobytes() + x.tobytes())
            sizes.append(rows), names.append("matvec_" + case[0])
        for case in RC.RMSNORM:
            n, eps, x, w = RC.rmsnorm_inputs(case)
            f.write(struct.pack("<2if", 2, n, eps) + x.tobytes() + w.tobytes())
            sizes.append(n), names.append("rmsnorm_" + case[0])
        for case in RC.ROPE:
            hd, nh, nkv, pos, base, q, k = RC.rope_inputs(case)
            f.write(struct.pack("<5if", 3, hd, nh, nkv, pos, base) + q.tobytes() + k.tobytes())
            sizes.append(q.size + k.size), names.append("rope_" + case[0])
        for case in RC.ATTN:
            hd, nh, nkv, n_past, max_ctx, q, kc, vc = RC.attn_inputs(case)
            f.write(struct.pack("<6i", 4, hd, nh, nkv, n_past, max_ctx) + q.tobytes() + kc.tobytes() + vc.tobytes())
            sizes.append(nh * hd), names.append("attention_" + case[0])
        for case in RC.SILU:
            n, g, u = RC.silu_inputs(case)
            f.write(struct.pack("<2i", 5, n) + g.tobytes() + u.tobytes())
            sizes.append(n), names.append("silu_" + case[0])
        f.write(struct.pack("<i", 0))
    subprocess.run([REF_ENGINE, "kernels", fin, fout], check=True)
    out = np.fromfile(fout, dtype=np.float32)
    assert out.size == sum(sizes), (out.size, sum(sizes))
    res, o = {}, 0
    for name, n in zip(names, sizes):
        res[name] = out[o:o + n].copy()
        o += n
    return res


def main() -> None:
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden", "ref_engine_c1.npz")
    with tempfile.TemporaryDirectory() as d:
        data = decode(d)
        data.update(kernels(d))
    np.savez_compressed(out, **data)
    print(f"wrote {out}: {len(data)} arrays; C1 tokens {data['c1_tokens'][16:].tolist()}")
    if len(sys.argv) > 2:
        subprocess.run([REF_ENGINE, "gemv", sys.argv[2]], check=True)
        print(open(sys.argv[2]).read())


if __name__ == "__main__":
    main()
