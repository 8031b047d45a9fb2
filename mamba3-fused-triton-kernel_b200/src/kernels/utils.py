"""PyTorch reference math of the Mamba-3 decode step.

Public helpers of the reference's ``src/kernels/utils.py`` (its tests import
them as ground truth, and ``Mamba3.step`` is built on them).  They are plain
PyTorch, run on any device, and are not used by the CUDA backends.
"""

import torch


def build_rope_freqs(num_angles: int, device: torch.device) -> torch.Tensor:
    """Inverse RoPE frequencies 1 / 10000^(i / num_angles), i < num_angles
    (reference: src/kernels/utils.py:19-28)."""
    i = torch.arange(num_angles, device=device, dtype=torch.float32)
    return torch.reciprocal(torch.pow(10000.0, i / num_angles))


def apply_rope(x: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (x[..., 2i], x[..., 2i+1]) by angles[..., i]
    (reference: src/kernels/utils.py:31-44)."""
    pairs = x.unflatten(-1, (-1, 2))
    even, odd = pairs[..., 0], pairs[..., 1]
    c, s = torch.cos(angles), torch.sin(angles)
    return torch.stack((even * c - odd * s, even * s + odd * c), dim=-1).flatten(-2)


def trapezoidal_blend(Bx_curr: torch.Tensor, Bx_prev: torch.Tensor,
                      trap: torch.Tensor) -> torch.Tensor:
    """(1 - trap) * Bx_curr + trap * 0.5 * (Bx_curr + Bx_prev): trap = 0 is
    the Euler step, trap = 1 the trapezoid (reference: src/kernels/utils.py:51-66)."""
    return (1.0 - trap) * Bx_curr + trap * 0.5 * (Bx_curr + Bx_prev)


def mamba3_siso_decode_ref(x, B_proj, C_proj, ADT, DT, trap, D_skip, h, bx_prev):
    """SISO state update + readout (reference: src/kernels/utils.py:73-102).

    x (B,H,P); B_proj, C_proj (B,H,D); ADT, DT, trap (B,H); D_skip (H,);
    h, bx_prev (B,H,P,D).  Returns new tensors (y (B,H,P), h, Bx) where Bx is
    the current, unblended x B^T that the next step blends with.
    """
    xf = x.float()
    bx = torch.einsum("bhp,bhd->bhpd", xf, B_proj.float())
    blend = trapezoidal_blend(bx, bx_prev.float(), trap[..., None, None])
    h_new = torch.exp(ADT)[..., None, None] * h.float() + DT[..., None, None] * blend
    y = torch.einsum("bhd,bhpd->bhp", C_proj.float(), h_new)
    y = y + D_skip[None, :, None] * xf
    return y, h_new, bx


def mamba3_mimo_decode_ref(x, B_proj, C_proj, ADT, DT, trap, D_skip, mimo_x, mimo_o,
                           h, bx_prev):
    """MIMO state update + readout (reference: src/kernels/utils.py:109-148).

    x (B,H,P); B_proj, C_proj (B,R,H,D); ADT, DT, trap (B,H); D_skip (H,);
    mimo_x, mimo_o (H,R,P); h, bx_prev (B,H,D).
    """
    x_r = torch.einsum("bhp,hrp->bhr", x.float(), mimo_x.float())
    bx = torch.einsum("bhr,brhd->bhd", x_r, B_proj.float())
    blend = trapezoidal_blend(bx, bx_prev.float(), trap[..., None])
    h_new = torch.exp(ADT)[..., None] * h.float() + DT[..., None] * blend
    y_r = torch.einsum("brhd,bhd->brh", C_proj.float(), h_new)
    y_r = y_r + D_skip[None, None, :] * x_r.transpose(1, 2)
    y = torch.einsum("brh,hrp->bhp", y_r, mimo_o.float())
    return y, h_new, bx


def _get_strides(shape: tuple, contiguous: bool = True) -> list:
    """Row-major element strides of ``shape`` (reference: src/kernels/utils.py:155-163)."""
    if not contiguous:
        raise ValueError("Only contiguous strides are supported")
    strides, acc = [], 1
    for s in reversed(shape):
        strides.append(acc)
        acc *= s
    return strides[::-1]
