"""Decode kernels (CUDA, sm_100a) and their PyTorch reference math.

Same module layout and names as the reference's ``src/kernels`` package.
"""

from src.kernels.siso_decode import mamba3_siso_decode_triton
from src.kernels.mimo_decode import mamba3_mimo_decode_triton
from src.kernels.siso_decode_fused import mamba3_siso_decode_fused_triton
from src.kernels.mimo_decode_fused import mamba3_mimo_decode_fused_triton
from src.kernels.fused_full_decode import (
    mamba3_mimo_full_fused_triton,
    mamba3_siso_full_fused_triton,
)
from src.kernels.utils import (
    apply_rope,
    build_rope_freqs,
    mamba3_mimo_decode_ref,
    mamba3_siso_decode_ref,
    trapezoidal_blend,
)
