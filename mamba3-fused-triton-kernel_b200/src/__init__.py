"""B200-native Mamba-3 single-token decode.

Drop-in replacement for the ``src`` package of
michaelYZh/mamba3-fused-triton-kernel: same module paths
(``src.models.inference.Mamba3Decoder``, ``src.models.mamba3.Mamba3``,
``src.kernels.*``) and the same public names, with every GPU routine
implemented as hand-written CUDA for sm_100a behind the C ABI declared in
``include/mamba3_b200.h`` (loaded from ``lib/libmamba3_b200.so``).
"""

from src.kernels import (
    apply_rope,
    build_rope_freqs,
    mamba3_mimo_decode_ref,
    mamba3_mimo_decode_triton,
    mamba3_siso_decode_ref,
    mamba3_siso_decode_triton,
    trapezoidal_blend,
)
from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3, MambaBlock, RMSNorm

__version__ = "1.0.0"
