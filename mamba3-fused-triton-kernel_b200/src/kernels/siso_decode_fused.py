"""SISO single-step decode with the silu(z) gate, on the sm_100a library.

Drop-in for the reference's ``src/kernels/siso_decode_fused.py``
(``m3_siso_decode_fused`` entry point of include/mamba3_b200.h).
"""

import torch

from src.kernels import _launch


def mamba3_siso_decode_fused_triton(
    x: torch.Tensor,        # (B, H, P)
    B_proj: torch.Tensor,   # (B, H, D)
    C_proj: torch.Tensor,   # (B, H, D)
    ADT: torch.Tensor,      # (B, H)
    DT: torch.Tensor,       # (B, H)
    trap: torch.Tensor,     # (B, H)
    D_skip: torch.Tensor,   # (H,)
    z_gate: torch.Tensor,   # (B, H, P)
    h: torch.Tensor,        # (B, H, P, D) float32, contiguous, updated in place
    bx_prev: torch.Tensor,  # (B, H, P, D) float32, contiguous, updated in place
) -> tuple:
    """SISO step with y * silu(z) applied in the kernel
    (reference: src/kernels/siso_decode_fused.py:143-193).

    Returns (y_gated, h, bx_prev).
    """
    B_dim, H_dim, P_dim = x.shape
    D_dim = B_proj.shape[-1]
    assert h.shape == (B_dim, H_dim, P_dim, D_dim)
    assert bx_prev.shape == (B_dim, H_dim, P_dim, D_dim)
    assert z_gate.shape == (B_dim, H_dim, P_dim)
    assert x.is_cuda and h.is_cuda
    y = _launch.ssm_decode(False, x, B_proj, C_proj, ADT, DT, trap, D_skip, h, bx_prev, z=z_gate)
    return y, h, bx_prev
