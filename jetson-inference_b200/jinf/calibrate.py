"""Activation profiling for the static predictor (reference tools/profile_activations.cpp).

    python -m jinf.calibrate --model model.nvmw [--output activations.bin] [--samples N]
                             [--threshold F]

Runs `samples` prompts of 8..31 random tokens (libc srand(42) / rand(), the reference tool's
generator, so the prompts are the same token sequences), counts on the GPU for every layer and
FFN neuron the tokens on which |SiLU(gate)| > threshold, and writes the frequencies in the
reference's profile format. jinf_engine_config.predictor_path (Engine(..., predictor_path=))
reads it back: the neurons with frequency > sparsity_threshold then run as the sparse FFN.
"""
import argparse
import ctypes as C

import numpy as np

from . import _lib as L
from .model import Engine


def reference_prompts(n_samples: int, n_vocab: int):
    """The reference tool's calibration prompts: srand(42); length 8 + rand() % 24, tokens
    rand() % n_vocab (reference tools/profile_activations.cpp:112-118)."""
    libc = C.CDLL(None)
    libc.rand.restype = C.c_int
    libc.srand(42)
    for _ in range(n_samples):
        n = 8 + libc.rand() % 24
        yield [libc.rand() % n_vocab for _ in range(n)]


def profile(engine: Engine, prompts, threshold: float):
    """Counts [n_layers, n_ff] and the number of tokens, one engine reset per prompt."""
    info = engine.h.contents
    counts = np.zeros((info.n_layers, info.n_ff), dtype=np.int32)
    total = 0
    for toks in prompts:
        engine.count_activations(toks, threshold, counts)
        total += len(toks)
        engine.reset()
    return counts, total


def write_profile(path: str, counts: np.ndarray, total_tokens: int) -> None:
    c = np.ascontiguousarray(counts, dtype=np.int32)
    L.check(L.lib.jinf_activation_profile_write(path.encode(), c.shape[0], c.shape[1], total_tokens,
                                                c.ctypes.data_as(C.c_void_p)), "jinf_activation_profile_write")


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", required=True)
    ap.add_argument("--output", default="activations.bin")
    ap.add_argument("--samples", type=int, default=1000)
    ap.add_argument("--threshold", type=float, default=0.1)
    a = ap.parse_args()
    eng = Engine.from_nvmw(a.model, max_context=64)
    counts, total = profile(eng, reference_prompts(a.samples, eng.h.contents.n_vocab), a.threshold)
    write_profile(a.output, counts, total)
    print(f"activation profile written to {a.output}: {total} tokens")


if __name__ == "__main__":
    main()
