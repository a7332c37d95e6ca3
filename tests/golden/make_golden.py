"""Generate the golden vectors under tests/golden/ from the REFERENCE's own code.

The reference's host sources (src/quant.cpp, src/gguf.cpp, src/splitter.cpp) are compiled
unmodified from its source tree into oracle/_ref/libjinf_ref.so by oracle/Makefile; this
script runs them on seeded inputs and stores inputs + outputs. The tests then pin both
the CPU oracle and the GPU kernels to these files, so they hold on machines without the
reference tree.

    python tests/golden/make_golden.py        # needs the reference tree (oracle/_ref)
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "jetson-inference_b200"))

from oracle import oracle  # noqa: E402

SPECIAL_F16 = [0x0000, 0x8000, 0x0001, 0x03ff, 0x0400, 0x3c00, 0xbc00, 0x7bff, 0xfbff, 0x7c00, 0xfc00, 0x7e00,
               0x3555, 0x2e66, 0x1234, 0x8abc]


def blocks(kind: str, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    bb = {"q4_0": 18, "q8_0": 34, "q4_K": 144}[kind]
    b = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    # fp16 scales: mostly realistic magnitudes, the first blocks carry special values
    d = (rng.standard_normal(n) * 0.002).astype(np.float16).view(np.uint16)
    d[: len(SPECIAL_F16)] = SPECIAL_F16
    b[:, 0] = d & 0xFF
    b[:, 1] = d >> 8
    if kind == "q4_K":
        dm = (np.abs(rng.standard_normal(n)) * 0.001).astype(np.float16).view(np.uint16)
        dm[: len(SPECIAL_F16)] = SPECIAL_F16[::-1]
        b[:, 2] = dm & 0xFF
        b[:, 3] = dm >> 8
    return b


def main() -> None:
    ref = oracle.ref_lib()
    if ref is None:
        raise SystemExit("reference library not available (oracle/_ref); cannot regenerate golden vectors")
    out = {}
    for kind, n, fn, per in [("q4_0", 256, ref.ref_dequantize_q4_0, 32), ("q8_0", 128, ref.ref_dequantize_q8_0, 32),
                             ("q4_K", 64, ref.ref_dequantize_q4_K, 256)]:
        b = blocks(kind, n, seed={"q4_0": 1, "q8_0": 2, "q4_K": 3}[kind])
        y = np.empty(n * per, dtype=np.float32)
        fn(b.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p), n)
        out[f"{kind}_blocks"] = b
        out[f"{kind}_out"] = y
    # every fp16 value through the reference's F16 path of jinf_dequantize
    h = np.arange(65536, dtype=np.uint16)
    f = np.empty(65536, dtype=np.float32)
    ref.ref_dequantize(h.ctypes.data_as(C.c_void_p), 1, f.ctypes.data_as(C.c_void_p), 65536)
    out["f16_all_sha256"] = np.frombuffer(hashlib.sha256(f.tobytes()).digest(), dtype=np.uint8)
    out["f16_sample_in"] = h[::257].copy()
    out["f16_sample_out"] = f[::257].copy()
    np.savez_compressed(os.path.join(HERE, "dequant_ref.npz"), **out)

    # GGUF parse + splitter placements of a synthetic model written by this library's writer
    import jinf
    shape = jinf.LlamaShape(2, 256, 4, 2, 512, 1024, 10000.0, 1e-5)
    m = jinf.SynthModel(shape, seed=7)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.gguf")
        m.write_gguf(path)
        buf = C.create_string_buffer(1 << 16)
        n = ref.ref_gguf_summary(path.encode(), buf, len(buf))
        lines = [buf.value[:n].decode()]
        nt = len(m.tensor_names())
        for budget in [0, 1 << 20, 2 << 20, 1 << 40]:
            pl = (C.c_int * nt)()
            tot = (C.c_ulonglong * 2)()
            cnt = ref.ref_split(path.encode(), budget, pl, tot)
            lines.append(f"split {budget} {cnt} {tot[0]} {tot[1]} " + "".join(str(pl[i]) for i in range(nt)) + "\n")
    with open(os.path.join(HERE, "gguf_split_ref.txt"), "w") as fh:
        fh.write("".join(lines))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
