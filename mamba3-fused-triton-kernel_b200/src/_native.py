"""ctypes binding of the sm_100a decode library (include/mamba3_b200.h).

The library is the only compute path of the CUDA backends: when it is
missing or cannot be loaded every CUDA entry point raises instead of falling
back to PyTorch.  Build it with ``python mamba3-fused-triton-kernel_b200/
build_native.py`` (or ``__graft_entry__.build()``).

Status codes from the library are mapped to the exception types the
reference raises for the same misuse: shape / dtype / alignment problems
become ``AssertionError`` (the reference asserts, e.g.
src/kernels/siso_decode.py:157-159) and an unsupported MIMO rank becomes
``ValueError`` (src/kernels/mimo_decode.py:426-430).
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_void_p

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "lib", "libmamba3_b200.so")

M3_F32, M3_BF16 = 0, 1
(M3_OK, M3_ERR_NULL, M3_ERR_SHAPE, M3_ERR_RANK, M3_ERR_DTYPE, M3_ERR_ALIGN, M3_ERR_LAUNCH, M3_ERR_DEVICE,
 M3_ERR_UNSUPPORTED, M3_ERR_SCRATCH) = range(10)
STEP_STATIC_SCRATCH_BYTES = 4 * 1024 * 1024  # M3_STEP_STATIC_SCRATCH_BYTES

SUPPORTED_RANKS = (1, 2, 4, 8)
MAX_D_STATE = 256


class Dims(ctypes.Structure):
    _fields_ = [("batch", c_int32), ("nheads", c_int32), ("headdim", c_int32),
                ("d_state", c_int32), ("mimo_rank", c_int32), ("num_rope_angles", c_int32),
                ("ngroups", c_int32), ("d_inner", c_int32), ("A_floor", c_float)]


class SsmArgs(ctypes.Structure):
    _fields_ = (
        [("x", c_void_p), ("x_sb", c_int64), ("x_sh", c_int64), ("x_sp", c_int64), ("x_dtype", c_int32),
         ("z", c_void_p), ("z_sb", c_int64), ("z_sh", c_int64), ("z_sp", c_int64), ("z_dtype", c_int32),
         ("y", c_void_p), ("y_sb", c_int64), ("y_sh", c_int64), ("y_sp", c_int64), ("y_dtype", c_int32),
         ("B_proj", c_void_p), ("B_sb", c_int64), ("B_sr", c_int64), ("B_sh", c_int64), ("B_sd", c_int64),
         ("C_proj", c_void_p), ("C_sb", c_int64), ("C_sr", c_int64), ("C_sh", c_int64), ("C_sd", c_int64),
         ("ADT", c_void_p), ("adt_sb", c_int64), ("adt_sh", c_int64),
         ("DT", c_void_p), ("dt_sb", c_int64), ("dt_sh", c_int64),
         ("trap", c_void_p), ("trap_sb", c_int64), ("trap_sh", c_int64),
         ("D_skip", c_void_p), ("D_sh", c_int64),
         ("mimo_x", c_void_p), ("mx_sh", c_int64), ("mx_sr", c_int64), ("mx_sp", c_int64),
         ("mimo_o", c_void_p), ("mo_sh", c_int64), ("mo_sr", c_int64), ("mo_sp", c_int64),
         ("h", c_void_p), ("bx_prev", c_void_p)])


class FullArgs(ctypes.Structure):
    _fields_ = [("zx", c_void_p), ("zx_stride_b", c_int64), ("zx_dtype", c_int32),
                ("param_dtype", c_int32),
                ("dt_bias", c_void_p), ("D", c_void_p), ("B_norm_w", c_void_p), ("C_norm_w", c_void_p),
                ("B_bias", c_void_p), ("C_bias", c_void_p), ("mimo_x", c_void_p), ("mimo_o", c_void_p),
                ("ssm_state", c_void_p), ("bx_prev", c_void_p), ("angle_state", c_void_p),
                ("y", c_void_p), ("y_stride_b", c_int64), ("y_dtype", c_int32)]


class StepArgs(ctypes.Structure):
    _fields_ = [("d_model", c_int32), ("dtype", c_int32),
                ("u", c_void_p), ("u_stride_b", c_int64),
                ("in_proj_w", c_void_p), ("in_proj_stride", c_int64),
                ("out_proj_w", c_void_p), ("out_proj_stride", c_int64),
                ("dt_bias", c_void_p), ("D", c_void_p), ("B_norm_w", c_void_p), ("C_norm_w", c_void_p),
                ("B_bias", c_void_p), ("C_bias", c_void_p), ("mimo_x", c_void_p), ("mimo_o", c_void_p),
                ("ssm_state", c_void_p), ("bx_prev", c_void_p), ("angle_state", c_void_p),
                ("out", c_void_p), ("out_stride_b", c_int64),
                ("workspace", c_void_p), ("workspace_bytes", c_int64)]


ENTRY_POINTS = {
    "m3_siso_decode": SsmArgs, "m3_mimo_decode": SsmArgs,
    "m3_siso_decode_fused": SsmArgs, "m3_mimo_decode_fused": SsmArgs,
    "m3_siso_full_fused": FullArgs, "m3_mimo_full_fused": FullArgs,
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """Load (once) and return the ctypes handle of the decode library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"the sm_100a decode library is not built ({path} missing); run "
                "`python mamba3-fused-triton-kernel_b200/build_native.py`")
        lib = ctypes.CDLL(path)
        for name, argt in ENTRY_POINTS.items():
            fn = getattr(lib, name)
            fn.argtypes = [POINTER(Dims), POINTER(argt), c_void_p]
            fn.restype = c_int
        lib.m3_linear_f32.argtypes = [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                      c_int32, c_int32, c_int32, c_void_p]
        lib.m3_linear_f32.restype = c_int
        lib.m3_linear_bf16.argtypes = [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                       c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p]
        lib.m3_linear_bf16.restype = c_int
        lib.m3_linear_bf16_workspace_bytes.argtypes = [c_int32, c_int32, c_int32]
        lib.m3_linear_bf16_workspace_bytes.restype = c_int64
        lib.m3_linear_f32_tc.argtypes = [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
                                         c_int64, c_int32, c_int32, c_int32, c_void_p]
        lib.m3_linear_f32_tc.restype = c_int
        lib.m3_split_tf32.argtypes = [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p]
        lib.m3_split_tf32.restype = c_int
        lib.m3_linear_bf16_skinny.argtypes = [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                              c_int32, c_int32, c_int32, c_int32, c_void_p]
        lib.m3_linear_bf16_skinny.restype = c_int
        lib.m3_mimo_prefill.argtypes = [POINTER(Dims), POINTER(FullArgs), c_int32, c_void_p]
        lib.m3_mimo_prefill.restype = c_int
        lib.m3_siso_prefill.argtypes = [POINTER(Dims), POINTER(FullArgs), c_int32, c_void_p]
        lib.m3_siso_prefill.restype = c_int
        lib.m3_residual_rmsnorm.argtypes = [c_int32, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
                                            c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32,
                                            c_float, c_void_p]
        lib.m3_residual_rmsnorm.restype = c_int
        lib.m3_mimo_step_workspace_bytes.argtypes = [POINTER(Dims), c_int32, c_int32]
        lib.m3_mimo_step_workspace_bytes.restype = c_int64
        lib.m3_mimo_step.argtypes = [POINTER(Dims), POINTER(StepArgs), c_void_p]
        lib.m3_mimo_step.restype = c_int
        lib.m3_siso_step_workspace_bytes.argtypes = [POINTER(Dims), c_int32, c_int32]
        lib.m3_siso_step_workspace_bytes.restype = c_int64
        lib.m3_siso_step.argtypes = [POINTER(Dims), POINTER(StepArgs), c_void_p]
        lib.m3_siso_step.restype = c_int
        lib.m3_mimo_step_static.argtypes = [POINTER(Dims), POINTER(StepArgs), c_void_p]
        lib.m3_mimo_step_static.restype = c_int
        lib.m3_device_error.argtypes = [c_int]
        lib.m3_device_error.restype = c_int
        lib.m3_selftest_wait_timeout.argtypes = [c_void_p]
        lib.m3_selftest_wait_timeout.restype = c_int
        lib.m3_version.argtypes = []
        lib.m3_version.restype = c_int
        lib.m3_status_string.argtypes = [c_int]
        lib.m3_status_string.restype = ctypes.c_char_p
        _lib = lib
    return _lib


M3_DEVERR_TIMEOUT = 1


def device_error(reset: bool = False) -> int:
    """Device error word of the library's kernels (synchronises the device):
    0, or M3_DEVERR_* bits of kernels that gave up a bounded wait."""
    return load().m3_device_error(1 if reset else 0)


def status_string(status: int) -> str:
    return load().m3_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status == M3_OK:
        return
    msg = f"{what}: {status_string(status)} (status {status})"
    if status == M3_ERR_RANK:
        raise ValueError(msg)
    if status in (M3_ERR_NULL, M3_ERR_SHAPE, M3_ERR_DTYPE, M3_ERR_ALIGN):
        raise AssertionError(msg)
    raise RuntimeError(msg)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return M3_F32
    if t.dtype == torch.bfloat16:
        return M3_BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def require_cuda_available(what: str = "the CUDA decode backend") -> None:
    if not torch.cuda.is_available():
        raise RuntimeError(f"{what} needs a CUDA device; none is available "
                           "(pass use_triton=False for the PyTorch reference path)")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class device_guard:
    """Make ``device`` current for the library call if it is not already."""

    __slots__ = ("dev", "prev")

    def __init__(self, device: torch.device):
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False
