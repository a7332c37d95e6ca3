"""jinf-b200: B200-native (sm_100a) implementation of the jetson-inference ("jinf")
per-token decode loop behind the reference's C-ABI.

Everything computes on the GPU through libjinf_b200.so (built in-tree); this package is
the host-side mirror of the reference's engine / kernel / loader interfaces.
"""
from . import _lib  # noqa: F401  (loads the library, fails loudly if it is missing)
from ._lib import F16, F32, Q4_0, Q4_K, Q6_K, Q8_0, JinfError, lib  # noqa: F401
from .model import LLAMA3_70B, LLAMA3_8B, TINY, Engine, LlamaShape, SynthModel, b200_options, nccl_unique_id  # noqa: F401
from . import kernels  # noqa: F401
