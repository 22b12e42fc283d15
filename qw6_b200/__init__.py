"""qw6_b200 -- B200-native replacement of qw6's quantized-matvec / MoE path.

The product is the C-ABI library ``libqw6cuda.so`` (include/qw6_vk.h,
include/qw6_cuda.h); this package holds its CUDA sources (csrc/), the ctypes
binding (lib.py) and the seeded synthetic-input generator (synth.py).
"""
from . import synth  # noqa: F401
from .lib import (  # noqa: F401
    BLOCK_BYTES, IQ2_S, IQ2_XXS, IQ3_S, LIB_PATH, Q4_K, Q5_K, Q6_K, Context, ExpertPack, Qw6CudaError, build,
    load,
)
