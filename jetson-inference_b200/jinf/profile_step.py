"""One persistent decode step of a 4-layer Llama-3-8B-shaped model (32k vocabulary) on
cuda:0, the small case used for full ncu captures of the step kernel.

    python -m jinf.profile_step [decode_steps]      (from jetson-inference_b200/)

The model holds ~0.6 GB of weights plus a 0.5 GB embedding table; the captured launch is
the 4th (prompt of 3 tokens, KV cache filled to position 512, one forwarded token).
"""
import sys


def main(steps: int = 4) -> None:
    import torch
    import jinf
    shape = jinf.LlamaShape(4, 4096, 32, 8, 14336, 32000, 5e5)
    eng = jinf.Engine.from_synth(jinf.SynthModel(shape, seed=0), max_context=600,
                                 options=jinf.b200_options(eos_token=-1))
    eng.forward([1, 2, 3])
    eng.fill_kv_random(512, seed=1)
    eng.forward([5])
    eng.decode_resident(steps)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 4)
