"""Full-step fused decode (everything between in_proj and out_proj) on the
sm_100a library.

Drop-in for the reference's ``src/kernels/fused_full_decode.py``: one kernel
launch does the split of the in_proj output, softplus(dt + dt_bias), the A
expression, sigmoid(trap), the angle-state accumulation, RMSNorm + bias +
RoPE on B/C, the exponential-trapezoidal state update, the C.h readout (MIMO:
rank-R down/up projections) and the silu(z) gate, updating ssm_state,
bx_prev and angle_state in place (``m3_siso_full_fused`` /
``m3_mimo_full_fused`` in include/mamba3_b200.h).
"""

import torch

from src.kernels import _launch


def mamba3_siso_full_fused_triton(
    zxBCdtAtrap: torch.Tensor,    # (B, d_in_proj) raw in_proj output
    dt_bias: torch.Tensor,        # (H,)
    D_skip: torch.Tensor,         # (H,)
    B_norm_weight: torch.Tensor,  # (D,)
    C_norm_weight: torch.Tensor,  # (D,)
    B_bias: torch.Tensor,         # (H, D)
    C_bias: torch.Tensor,         # (H, D)
    h: torch.Tensor,              # (B, H, P, D) float32, in place
    bx_prev: torch.Tensor,        # (B, H, P, D) float32, in place
    angle_state: torch.Tensor,    # (B, H, num_rope_angles) float32, in place
    d_inner: int,
    d_state: int,
    ngroups: int,
    mimo_rank: int,
    nheads: int,
    headdim: int,
    split_tensor_size: int,
    num_rope_angles: int,
    A_floor: float,
) -> tuple:
    """SISO full decode step (reference: src/kernels/fused_full_decode.py:228-289).

    Returns (y_gated (B, H, P) float32, h, bx_prev, angle_state).
    """
    B_batch = zxBCdtAtrap.shape[0]
    H, P, D = nheads, headdim, d_state
    assert h.shape == (B_batch, H, P, D)
    assert bx_prev.shape == (B_batch, H, P, D)
    assert angle_state.shape == (B_batch, H, num_rope_angles)
    assert zxBCdtAtrap.is_cuda and h.is_cuda
    y = _launch.full_fused(
        False, zxBCdtAtrap, dt_bias, D_skip, B_norm_weight, C_norm_weight, B_bias, C_bias,
        None, None, h, bx_prev, angle_state, d_inner=d_inner, d_state=d_state, ngroups=ngroups,
        mimo_rank=1, nheads=nheads, headdim=headdim, split_tensor_size=split_tensor_size,
        num_rope_angles=num_rope_angles, A_floor=A_floor)
    return y, h, bx_prev, angle_state


def mamba3_mimo_full_fused_triton(
    zxBCdtAtrap: torch.Tensor,    # (B, d_in_proj) raw in_proj output
    dt_bias: torch.Tensor,        # (H,)
    D_skip: torch.Tensor,         # (H,)
    B_norm_weight: torch.Tensor,  # (D,)
    C_norm_weight: torch.Tensor,  # (D,)
    B_bias: torch.Tensor,         # (H, R, D)
    C_bias: torch.Tensor,         # (H, R, D)
    mimo_x: torch.Tensor,         # (H, R, P)
    mimo_o: torch.Tensor,         # (H, R, P)
    h: torch.Tensor,              # (B, H, D) float32, in place
    bx_prev: torch.Tensor,        # (B, H, D) float32, in place
    angle_state: torch.Tensor,    # (B, H, num_rope_angles) float32, in place
    d_inner: int,
    d_state: int,
    ngroups: int,
    mimo_rank: int,
    nheads: int,
    headdim: int,
    split_tensor_size: int,
    num_rope_angles: int,
    A_floor: float,
) -> tuple:
    """MIMO full decode step (reference: src/kernels/fused_full_decode.py:569-636).

    The reference kernel exists for R == 4 only; this one serves R in
    {1, 2, 4, 8} and raises ValueError for any other rank.

    Returns (y_gated (B, H, P) float32, h, bx_prev, angle_state).
    """
    B_batch = zxBCdtAtrap.shape[0]
    H, D = nheads, d_state
    assert h.shape == (B_batch, H, D)
    assert bx_prev.shape == (B_batch, H, D)
    assert angle_state.shape == (B_batch, H, num_rope_angles)
    assert zxBCdtAtrap.is_cuda and h.is_cuda
    y = _launch.full_fused(
        True, zxBCdtAtrap, dt_bias, D_skip, B_norm_weight, C_norm_weight, B_bias, C_bias,
        mimo_x, mimo_o, h, bx_prev, angle_state, d_inner=d_inner, d_state=d_state,
        ngroups=ngroups, mimo_rank=mimo_rank, nheads=nheads, headdim=headdim,
        split_tensor_size=split_tensor_size, num_rope_angles=num_rope_angles, A_floor=A_floor)
    return y, h, bx_prev, angle_state
