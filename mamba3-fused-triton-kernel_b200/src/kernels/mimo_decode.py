"""MIMO single-step decode on the sm_100a library.

Drop-in for the reference's ``src/kernels/mimo_decode.py``
(``m3_mimo_decode`` entry point of include/mamba3_b200.h).  Ranks 1, 2, 4
and 8 are supported, as in the reference; any other rank raises ValueError.
"""

import torch

from src.kernels import _launch
from src._native import SUPPORTED_RANKS


def mamba3_mimo_decode_triton(
    x: torch.Tensor,        # (B, H, P)
    B_proj: torch.Tensor,   # (B, R, H, D)
    C_proj: torch.Tensor,   # (B, R, H, D)
    ADT: torch.Tensor,      # (B, H)
    DT: torch.Tensor,       # (B, H)
    trap: torch.Tensor,     # (B, H)
    D_skip: torch.Tensor,   # (H,)
    mimo_x: torch.Tensor,   # (H, R, P)
    mimo_o: torch.Tensor,   # (H, R, P)
    h: torch.Tensor,        # (B, H, D) float32, contiguous, updated in place
    bx_prev: torch.Tensor,  # (B, H, D) float32, contiguous, updated in place
) -> tuple:
    """One MIMO state update + readout (reference: src/kernels/mimo_decode.py:394-457).

    x_r = mimo_x x;  Bx = sum_r x_r B_r;  trapezoidal update of h;
    y_r = C_r h + D_skip x_r;  y = sum_r y_r mimo_o[:, r].

    Returns (y, h, bx_prev); y is a new tensor like ``x``.
    """
    B_dim, H_dim, P_dim = x.shape
    R_dim = B_proj.shape[1]
    D_dim = B_proj.shape[-1]
    assert h.shape == (B_dim, H_dim, D_dim)
    assert bx_prev.shape == (B_dim, H_dim, D_dim)
    assert mimo_x.shape == (H_dim, R_dim, P_dim)
    assert mimo_o.shape == (H_dim, R_dim, P_dim)
    assert x.is_cuda and h.is_cuda
    if R_dim not in SUPPORTED_RANKS:
        raise ValueError(
            f"Unsupported mimo_rank={R_dim}. Supported values: {list(SUPPORTED_RANKS)}")
    y = _launch.ssm_decode(True, x, B_proj, C_proj, ADT, DT, trap, D_skip, h, bx_prev,
                           mimo_x=mimo_x, mimo_o=mimo_o)
    return y, h, bx_prev
