"""The decode step's projections (in_proj / out_proj) on the GPU.

``linear(x, weight)`` computes ``x @ weight.T`` (``nn.Linear`` without bias,
src/models/mamba3.py:115,158).  Small fp32 batches -- the latency-bound
decode regime -- run the library's ``m3_linear_f32`` kernel; larger batches
and bf16 use cuBLAS through ``torch.nn.functional.linear``, where tensor
cores or large tiles pay.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from src import _native as nat

SMALL_M_MAX = 256  # batch rows up to which the latency-optimised kernel is used


def uses_small_m_kernel(x: torch.Tensor, weight: torch.Tensor) -> bool:
    return (x.is_cuda and x.dim() == 2 and x.dtype == torch.float32 and weight.dtype == torch.float32
            and x.shape[0] <= SMALL_M_MAX and x.shape[1] % 4 == 0 and x.stride(1) == 1
            and weight.stride(1) == 1 and x.stride(0) % 4 == 0 and weight.stride(0) % 4 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0 and weight.device == x.device)


def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``x @ weight.T`` for x (M, K), weight (N, K)."""
    if not uses_small_m_kernel(x, weight):
        return F.linear(x, weight)
    M, K = x.shape
    N = weight.shape[0]
    assert weight.shape[1] == K, f"weight must be (N, {K}), got {tuple(weight.shape)}"
    out = torch.empty(M, N, device=x.device, dtype=torch.float32)
    if M == 0:
        return out
    with nat.device_guard(x.device):
        st = nat.load().m3_linear_f32(x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0),
                                      out.data_ptr(), out.stride(0), M, N, K, nat.stream_handle(x.device))
    nat.check(st, "m3_linear_f32")
    return out
