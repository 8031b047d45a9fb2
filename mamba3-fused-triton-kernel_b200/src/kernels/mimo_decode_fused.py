"""MIMO single-step decode with the silu(z) gate, on the sm_100a library.

Drop-in for the reference's ``src/kernels/mimo_decode_fused.py``
(``m3_mimo_decode_fused`` entry point of include/mamba3_b200.h).  The
reference supports only R == 4 here; this version accepts R in {1, 2, 4, 8}.
"""

import torch

from src.kernels import _launch
from src._native import SUPPORTED_RANKS


def mamba3_mimo_decode_fused_triton(
    x: torch.Tensor,        # (B, H, P)
    B_proj: torch.Tensor,   # (B, R, H, D)
    C_proj: torch.Tensor,   # (B, R, H, D)
    ADT: torch.Tensor,      # (B, H)
    DT: torch.Tensor,       # (B, H)
    trap: torch.Tensor,     # (B, H)
    D_skip: torch.Tensor,   # (H,)
    mimo_x: torch.Tensor,   # (H, R, P)
    mimo_o: torch.Tensor,   # (H, R, P)
    z_gate: torch.Tensor,   # (B, H, P)
    h: torch.Tensor,        # (B, H, D) float32, contiguous, updated in place
    bx_prev: torch.Tensor,  # (B, H, D) float32, contiguous, updated in place
) -> tuple:
    """MIMO step with y * silu(z) applied in the kernel
    (reference: src/kernels/mimo_decode_fused.py:114-170).

    Returns (y_gated, h, bx_prev).
    """
    B_dim = x.shape[0]
    H_dim = x.shape[1]
    P_dim = x.shape[2]
    R_dim = B_proj.shape[1]
    D_dim = B_proj.shape[-1]
    assert h.shape == (B_dim, H_dim, D_dim)
    assert bx_prev.shape == (B_dim, H_dim, D_dim)
    assert z_gate.shape == (B_dim, H_dim, P_dim)
    assert x.is_cuda and h.is_cuda
    if R_dim not in SUPPORTED_RANKS:
        raise ValueError(
            f"Unsupported mimo_rank={R_dim}. Supported values: {list(SUPPORTED_RANKS)}")
    y = _launch.ssm_decode(True, x, B_proj, C_proj, ADT, DT, trap, D_skip, h, bx_prev,
                           mimo_x=mimo_x, mimo_o=mimo_o, z=z_gate)
    return y, h, bx_prev
