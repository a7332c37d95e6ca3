"""GGUF -> NVMW conversion (reference tools/prepare_model; the same file byte for byte).

    python -m jinf.prepare_model --input model.gguf --output model.nvmw [--gpu-budget MB] [--bundled]
"""
import argparse

from . import _lib as L


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--input", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--gpu-budget", type=int, default=4500, help="MB (reference default 4500)")
    ap.add_argument("--bundled", action="store_true", help="write the neuron bundles of the sparse FFN")
    a = ap.parse_args()
    L.check(L.lib.jinf_prepare_model(a.input.encode(), a.output.encode(), a.gpu_budget, int(a.bundled)),
            "jinf_prepare_model")
    print(f"wrote {a.output}")


if __name__ == "__main__":
    main()
