"""GGUF -> NVMW conversion (reference tools/prepare_model; the same file byte for byte).

    python -m jinf.prepare_model --input model.gguf --output model.nvmw [--gpu-budget MB] [--bundled]
    python -m jinf.prepare_model --input model.gguf --output model.nvmw --b200 [--tp N]

--b200 writes the B200 layout instead (NVMW version 3, new): every projection pre-packed into
the engine's Q4M image, loaded without repacking, for the dense FFN on one GPU, or with --tp N
as N tensor-parallel shards (each rank's slice of every projection as an image of its own).
"""
import argparse

from . import _lib as L


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--input", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--gpu-budget", type=int, default=4500, help="MB (reference default 4500)")
    ap.add_argument("--bundled", action="store_true", help="write the neuron bundles of the sparse FFN")
    ap.add_argument("--b200", action="store_true", help="write the pre-packed B200 layout (version 3)")
    ap.add_argument("--tp", type=int, default=1, choices=[1, 2, 4, 8], help="--b200: tensor-parallel GPUs")
    a = ap.parse_args()
    if a.b200:
        L.check(L.lib.jinf_prepare_model_b200_tp(a.input.encode(), a.output.encode(), a.tp),
                "jinf_prepare_model_b200_tp")
    else:
        L.check(L.lib.jinf_prepare_model(a.input.encode(), a.output.encode(), a.gpu_budget, int(a.bundled)),
                "jinf_prepare_model")
    print(f"wrote {a.output}")


if __name__ == "__main__":
    main()
