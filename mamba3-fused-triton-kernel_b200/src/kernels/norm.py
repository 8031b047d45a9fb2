"""Residual add + RMSNorm between stacked blocks (``m3_residual_rmsnorm``).

``residual_rmsnorm(x, o, w)`` returns ``(x + o, RMSNorm_w(x + o))`` in x's
dtype with fp32 normalisation math, as the reference block
``x + mixer(norm(x))`` with ``RMSNorm`` computes them
(src/models/mamba3.py:26-36, 412-421); ``o=None`` normalises x alone.
"""

from __future__ import annotations

import torch

from src import _native as nat


def residual_rmsnorm(x: torch.Tensor, o: torch.Tensor | None, weight: torch.Tensor | None,
                     eps: float = 1e-5) -> tuple:
    """(x + o, RMSNorm_weight(x + o)); o=None skips the add, weight=None
    skips the norm (returning None in its place)."""
    assert x.is_cuda and x.dim() == 2 and x.stride(1) == 1
    assert o is not None or weight is not None
    M, N = x.shape
    if o is not None:
        assert o.shape == x.shape and o.dtype == x.dtype and o.stride(1) == 1 and o.device == x.device
    w = None
    if weight is not None:
        w = weight.detach().float().contiguous()
        assert w.shape == (N,) and w.device == x.device
    x_out = torch.empty_like(x) if o is not None else None
    xn = torch.empty_like(x) if w is not None else None
    if M > 0:
        with nat.device_guard(x.device):
            st = nat.load().m3_residual_rmsnorm(
                nat.dtype_code(x), x.data_ptr(), x.stride(0), None if o is None else o.data_ptr(),
                0 if o is None else o.stride(0), None if w is None else w.data_ptr(),
                None if x_out is None else x_out.data_ptr(), 0 if x_out is None else x_out.stride(0),
                None if xn is None else xn.data_ptr(), 0 if xn is None else xn.stride(0), M, N, float(eps),
                nat.stream_handle(x.device))
        nat.check(st, "m3_residual_rmsnorm")
    return (x_out if o is not None else x), xn
