"""The decode step's projections (in_proj / out_proj) on the GPU.

``linear(x, weight)`` computes ``x @ weight.T`` (``nn.Linear`` without bias,
src/models/mamba3.py:115,158).  Small fp32 batches -- the latency-bound
decode regime -- run the library's ``m3_linear_f32`` kernel; larger fp32
batches (on large layers from a few dozen rows) run the library's
split-precision tensor-core GEMM
(``m3_linear_f32_tc``: each operand split into a TF32 head and remainder,
three tcgen05 kind::tf32 products per k step, about fp32 accuracy; the
weight's split is computed once and cached); bf16 batches of up to
``SKINNY_ROUTE_M`` rows run the library's weight-streaming kernel
(``m3_linear_bf16_skinny``: 24 layers of the d_model 2048 stack's in_proj +
out_proj at 8 rows in 16.4 us a layer against cuBLAS's 21.1 us on B200;
from 32 rows cuBLAS is faster); with ``TC_ROUTE`` set, bf16 batches up to
``TC_MAX_M`` rows run the library's tcgen05 GEMM (``m3_linear_bf16``: pairs
of SMs sharing each batch tile, ``cta_group::2``); everything else uses
cuBLAS through ``torch.nn.functional.linear``.  ``TC_ROUTE`` is off: at the
decode shapes measured on B200 cuBLAS is faster (24 layers of in_proj +
out_proj at batch 256, d_model 2048: 473 us against 860 us).
"""

from __future__ import annotations

import weakref

import torch
import torch.nn.functional as F

from src import _native as nat

SMALL_M_MAX = 256  # batch rows up to which the latency-optimised kernel is used
TC_MAX_M = 512     # bf16 batch rows up to which TC_ROUTE uses the tcgen05 GEMM
TC_ROUTE = False   # route bf16 projections to m3_linear_bf16 (off: cuBLAS is faster at the decode shapes)
TF32X3_ROUTE = True  # route large fp32 projections to m3_linear_f32_tc
# fp32 batches of at most SMALL_M_MAX rows also take m3_linear_f32_tc on
# large layers (K and N >= 1024) once M x N reaches TF32X3_MIN_WORK and M
# TF32X3_MIN_ROWS: measured on B200 for the d_model 1024 layer, in_proj
# (N 4224-6272, K 1024) at 32 rows 30.7 against 41.0 us on the small-batch
# kernel and at 128 rows 34.8 against 116.7 us; out_proj (N 1024, K 2048)
# at 128 rows 49.2 against 53.3 us, at 64 rows 47.1 against 28.7 us
TF32X3_MIN_ROWS = 17
TF32X3_MIN_WORK = 1 << 17
SKINNY_MAX_M = 64    # bf16 batch rows up to which m3_linear_bf16_skinny applies
SKINNY_ROUTE_M = 16  # bf16 batch rows up to which linear() routes to it (cuBLAS is faster above)


def uses_small_m_kernel(x: torch.Tensor, weight: torch.Tensor) -> bool:
    return (x.is_cuda and x.dim() == 2 and x.dtype == torch.float32 and weight.dtype == torch.float32
            and x.shape[0] <= SMALL_M_MAX and x.shape[1] % 4 == 0 and x.stride(1) == 1
            and weight.stride(1) == 1 and x.stride(0) % 4 == 0 and weight.stride(0) % 4 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0 and weight.device == x.device)


def uses_tc_bf16(x: torch.Tensor, weight: torch.Tensor) -> bool:
    return (x.is_cuda and x.dim() == 2 and weight.dim() == 2 and x.dtype == torch.bfloat16
            and weight.dtype == torch.bfloat16 and 0 < x.shape[0] <= TC_MAX_M and x.shape[1] >= 64
            and x.shape[1] % 8 == 0 and weight.shape[1] == x.shape[1] and x.stride(1) == 1
            and weight.stride(1) == 1 and x.stride(0) % 8 == 0 and weight.stride(0) % 8 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0 and weight.device == x.device)


def uses_skinny_bf16(x: torch.Tensor, weight: torch.Tensor) -> bool:
    return (x.is_cuda and x.dim() == 2 and weight.dim() == 2 and x.dtype == torch.bfloat16
            and weight.dtype == torch.bfloat16 and 0 < x.shape[0] <= SKINNY_MAX_M and x.shape[1] > 0
            and x.shape[1] % 8 == 0 and weight.shape[1] == x.shape[1] and x.stride(1) == 1
            and weight.stride(1) == 1 and x.stride(0) % 8 == 0 and weight.stride(0) % 8 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0 and weight.device == x.device)


def uses_tf32x3(x: torch.Tensor, weight: torch.Tensor) -> bool:
    if x.dim() != 2 or weight.dim() != 2:
        return False
    M, K, N = x.shape[0], x.shape[1], weight.shape[0]
    big = M > SMALL_M_MAX or (M >= TF32X3_MIN_ROWS and M * N >= TF32X3_MIN_WORK and K >= 1024 and N >= 1024)
    return (big and x.is_cuda and x.dtype == torch.float32
            and weight.dtype == torch.float32 and x.shape[1] >= 32
            and x.shape[1] % 4 == 0 and weight.shape[1] == x.shape[1] and x.stride(1) == 1
            and weight.stride(1) == 1 and x.stride(0) % 4 == 0 and weight.stride(0) % 4 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0 and weight.device == x.device)


# id(weight) -> ((data_ptr, version, shape, stride), hi, lo); an entry is
# dropped when its weight tensor is freed, so a later tensor that reuses the
# memory (or the id) never meets a stale split
_weight_splits: dict = {}


def tf32_split(x: torch.Tensor):
    """(hi, lo): x with its 13 low mantissa bits cleared and the exact
    remainder, contiguous fp32 (m3_split_tf32)."""
    M, K = x.shape
    hi = torch.empty(M, K, device=x.device, dtype=torch.float32)
    lo = torch.empty_like(hi)
    with nat.device_guard(x.device):
        st = nat.load().m3_split_tf32(x.data_ptr(), x.stride(0), hi.data_ptr(), lo.data_ptr(), K, M, K,
                                      nat.stream_handle(x.device))
    nat.check(st, "m3_split_tf32")
    return hi, lo


def _weight_split(weight: torch.Tensor):
    """The weight's TF32 head and remainder, computed once per weight tensor
    (and again after an in-place change, which bumps its version).  A CUDA
    graph that captured a projection keeps using the split it captured, so a
    weight changed after capture needs a new capture."""
    k = id(weight)
    sig = (weight.device.index, weight.data_ptr(), weight._version, tuple(weight.shape), tuple(weight.stride()))
    hit = _weight_splits.get(k)
    if hit is not None and hit[0] == sig:
        return hit[1], hit[2]
    if hit is None:
        weakref.finalize(weight, _weight_splits.pop, k, None)
    hi, lo = tf32_split(weight)
    _weight_splits[k] = (sig, hi, lo)
    return hi, lo


def linear_tf32x3(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``x @ weight.T`` for fp32 x (M, K), weight (N, K) on the tensor cores
    in split precision (m3_linear_f32_tc)."""
    M, K = x.shape
    N = weight.shape[0]
    out = torch.empty(M, N, device=x.device, dtype=torch.float32)
    w_hi, w_lo = _weight_split(weight)
    x_hi, x_lo = tf32_split(x)
    with nat.device_guard(x.device):
        st = nat.load().m3_linear_f32_tc(x_hi.data_ptr(), x_lo.data_ptr(), K, w_hi.data_ptr(), w_lo.data_ptr(), K,
                                         out.data_ptr(), out.stride(0), M, N, K, nat.stream_handle(x.device))
    nat.check(st, "m3_linear_f32_tc")
    return out


_workspaces: dict = {}  # device index -> split-K workspace, grown on demand and kept


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """The device's split-K workspace, at least ``nbytes``, zeroed when it is
    allocated; the GEMM leaves what it used at zero again after every call.
    Calls on one device share it, which is safe because they run in stream
    order; it is kept for the life of the process (CUDA graphs that captured
    a call keep pointing at it), so the first calls of each shape should
    come before capture."""
    ws = _workspaces.get(device.index)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[device.index] = ws
    return ws


def linear_bf16(x: torch.Tensor, weight: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """``x @ weight.T`` on the tcgen05 GEMM (bf16 operands, fp32
    accumulation, output rounded to ``out_dtype``)."""
    M, K = x.shape
    N = weight.shape[0]
    out = torch.empty(M, N, device=x.device, dtype=out_dtype)
    code = nat.M3_BF16 if out_dtype == torch.bfloat16 else nat.M3_F32
    lib = nat.load()
    with nat.device_guard(x.device):
        need = lib.m3_linear_bf16_workspace_bytes(M, N, K)
        ws = _workspace(x.device, need) if need > 0 else None
        st = lib.m3_linear_bf16(x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0),
                                out.data_ptr(), out.stride(0), M, N, K, code,
                                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                                nat.stream_handle(x.device))
    nat.check(st, "m3_linear_bf16")
    return out


def linear_bf16_skinny(x: torch.Tensor, weight: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """``x @ weight.T`` for a bf16 batch of at most SKINNY_MAX_M rows on the
    weight-streaming kernel (fp32 accumulation, output rounded to
    ``out_dtype``)."""
    M, K = x.shape
    N = weight.shape[0]
    out = torch.empty(M, N, device=x.device, dtype=out_dtype)
    code = nat.M3_BF16 if out_dtype == torch.bfloat16 else nat.M3_F32
    with nat.device_guard(x.device):
        st = nat.load().m3_linear_bf16_skinny(x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0),
                                              out.data_ptr(), out.stride(0), M, N, K, code,
                                              nat.stream_handle(x.device))
    nat.check(st, "m3_linear_bf16_skinny")
    return out


def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``x @ weight.T`` for x (M, K), weight (N, K)."""
    if x.dim() == 2 and x.shape[0] <= SKINNY_ROUTE_M and uses_skinny_bf16(x, weight):
        return linear_bf16_skinny(x, weight)
    if TC_ROUTE and uses_tc_bf16(x, weight):
        return linear_bf16(x, weight)
    if TF32X3_ROUTE and uses_tf32x3(x, weight):
        return linear_tf32x3(x, weight)
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
