"""Regenerates tests/golden/prepare_model_ref.txt: the SHA-256 of the NVMW files that the
reference's own tools/prepare_model (compiled unmodified by oracle/Makefile into
oracle/_ref/prepare_model) writes from the synthetic tiny model's GGUF, for a hot/cold split
budget and with or without neuron bundles.

    python tests/golden/make_prepare_golden.py          (from the repository root)
"""
import hashlib
import os
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "jetson-inference_b200"))

CASES = [(4500, 0), (4500, 1), (8, 0), (8, 1)]  # (gpu budget MB, bundled)


def main() -> None:
    import jinf
    tool = os.path.join(ROOT, "oracle", "_ref", "prepare_model")
    with tempfile.TemporaryDirectory() as d:
        gguf = os.path.join(d, "tiny.gguf")
        jinf.SynthModel(jinf.TINY, seed=0).write_gguf(gguf)
        lines = []
        for budget, bundled in CASES:
            out = os.path.join(d, "ref.nvmw")
            cmd = [tool, "--input", gguf, "--output", out, "--gpu-budget", str(budget)] + (["--bundled"] if bundled else [])
            subprocess.run(cmd, check=True, capture_output=True)
            lines.append(f"{budget} {bundled} {os.path.getsize(out)} {hashlib.sha256(open(out, 'rb').read()).hexdigest()}")
    with open(os.path.join(ROOT, "tests", "golden", "prepare_model_ref.txt"), "w") as f:
        f.write("# gpu_budget_mb bundled bytes sha256 (reference tools/prepare_model on SynthModel(TINY, seed=0))\n")
        f.write("\n".join(lines) + "\n")


if __name__ == "__main__":
    main()
