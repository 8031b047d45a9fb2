"""SISO single-step decode on the sm_100a library.

Drop-in for the reference's ``src/kernels/siso_decode.py``: same function
name, arguments, in-place contract and return value; the GPU work is the
``m3_siso_decode`` entry point of include/mamba3_b200.h.
"""

import torch

from src.kernels import _launch


def mamba3_siso_decode_triton(
    x: torch.Tensor,        # (B, H, P)
    B_proj: torch.Tensor,   # (B, H, D)
    C_proj: torch.Tensor,   # (B, H, D)
    ADT: torch.Tensor,      # (B, H)
    DT: torch.Tensor,       # (B, H)
    trap: torch.Tensor,     # (B, H)
    D_skip: torch.Tensor,   # (H,)
    h: torch.Tensor,        # (B, H, P, D) float32, contiguous, updated in place
    bx_prev: torch.Tensor,  # (B, H, P, D) float32, contiguous, updated in place
) -> tuple:
    """One SISO state update + readout (reference: src/kernels/siso_decode.py:136-187).

    h <- exp(ADT) h + DT [(1-trap) Bx + trap/2 (Bx + bx_prev)],  Bx = x B^T,
    y = h C + D_skip x,  bx_prev <- Bx.

    Returns (y, h, bx_prev); y is a new tensor like ``x``.
    """
    B_dim, H_dim, P_dim = x.shape
    D_dim = B_proj.shape[-1]
    assert h.shape == (B_dim, H_dim, P_dim, D_dim)
    assert bx_prev.shape == (B_dim, H_dim, P_dim, D_dim)
    assert x.is_cuda and h.is_cuda
    y = _launch.ssm_decode(False, x, B_proj, C_proj, ADT, DT, trap, D_skip, h, bx_prev)
    return y, h, bx_prev
