"""C-ABI checks that need no GPU.

* the library loads and exports every function include/mamba3_b200.h declares;
* the ctypes structures match the C layout (gcc compiles the header and
  reports sizeof/offsetof);
* host-side validation rejects bad calls before touching a device.
"""

from __future__ import annotations

import ctypes
import os
import re
import subprocess
import tempfile

import pytest
import torch

from conftest import ROOT
from src import _native as nat

HEADER = os.path.join(ROOT, "include", "mamba3_b200.h")


def _declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char \*)\s*(m3_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = nat.load()
    names = _declared_functions()
    assert len(names) == 24, names
    for n in names:
        assert hasattr(lib, n), f"{n} not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", nat.LIB_PATH], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (m3_\w+)", out.stdout))
    assert set(names) <= exported
    assert lib.m3_version() == 10400
    assert nat.status_string(nat.M3_ERR_RANK).startswith("unsupported mimo_rank")


_LAYOUT_C = r"""
#include <stdio.h>
#include <stddef.h>
#include "mamba3_b200.h"
#define P(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("m3_dims %zu\nm3_ssm_args %zu\nm3_full_args %zu\nm3_step_args %zu\n",
         sizeof(m3_dims), sizeof(m3_ssm_args), sizeof(m3_full_args), sizeof(m3_step_args));
  P(m3_dims, A_floor) P(m3_ssm_args, z) P(m3_ssm_args, y_dtype) P(m3_ssm_args, B_sd)
  P(m3_ssm_args, trap_sh) P(m3_ssm_args, mo_sp) P(m3_ssm_args, bx_prev)
  P(m3_full_args, param_dtype) P(m3_full_args, mimo_o) P(m3_full_args, y_dtype)
  P(m3_step_args, u) P(m3_step_args, out_proj_stride) P(m3_step_args, mimo_o) P(m3_step_args, angle_state)
  P(m3_step_args, out_stride_b) P(m3_step_args, workspace_bytes)
  return 0;
}
"""


def test_ctypes_layout_matches_c_header():
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "l.c"), os.path.join(d, "l")
        open(src, "w").write(_LAYOUT_C)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), src, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.rsplit(" ", 1) for l in lines if l)
    assert int(got["m3_dims"]) == ctypes.sizeof(nat.Dims)
    assert int(got["m3_ssm_args"]) == ctypes.sizeof(nat.SsmArgs)
    assert int(got["m3_full_args"]) == ctypes.sizeof(nat.FullArgs)
    assert int(got["m3_step_args"]) == ctypes.sizeof(nat.StepArgs)
    pairs = {"m3_dims": nat.Dims, "m3_ssm_args": nat.SsmArgs, "m3_full_args": nat.FullArgs,
             "m3_step_args": nat.StepArgs}
    for key, val in got.items():
        if "." in key:
            struct, field = key.split(".")
            assert getattr(pairs[struct], field).offset == int(val), key


def _ssm_call(dims, args, mimo=False, fused=False):
    lib = nat.load()
    name = f"m3_{'mimo' if mimo else 'siso'}_decode{'_fused' if fused else ''}"
    return getattr(lib, name)(dims, args, None)


def _valid_ssm(mimo=False, fused=False):
    """Argument blocks with fake but well-aligned device addresses (the
    library never dereferences them on the host)."""
    dims = nat.Dims(batch=2, nheads=4, headdim=16, d_state=64, mimo_rank=4 if mimo else 1,
                    num_rope_angles=0, ngroups=1, d_inner=64, A_floor=0.0)
    a = nat.SsmArgs()
    fake = 0x7000_0000_0000
    for i, f in enumerate(["x", "y", "B_proj", "C_proj", "ADT", "DT", "trap", "D_skip", "h",
                           "bx_prev", "mimo_x", "mimo_o", "z"]):
        setattr(a, f, fake + 4096 * i)
    if not fused:
        a.z = None
    return dims, a


def test_validation_null_and_shape():
    lib = nat.load()
    assert lib.m3_siso_decode(None, None, None) == nat.M3_ERR_NULL
    dims, a = _valid_ssm()
    a.h = None
    assert _ssm_call(dims, a) == nat.M3_ERR_NULL
    for field, bad in [("d_state", 6), ("d_state", 512), ("headdim", 0), ("nheads", -1)]:
        dims, a = _valid_ssm()
        setattr(dims, field, bad)
        assert _ssm_call(dims, a) == nat.M3_ERR_SHAPE, (field, bad)


def test_validation_rank_dtype_alignment():
    dims, a = _valid_ssm(mimo=True)
    dims.mimo_rank = 3
    assert _ssm_call(dims, a, mimo=True) == nat.M3_ERR_RANK
    dims, a = _valid_ssm()
    a.x_dtype = 7
    assert _ssm_call(dims, a) == nat.M3_ERR_DTYPE
    dims, a = _valid_ssm()
    a.h = a.h + 4
    assert _ssm_call(dims, a) == nat.M3_ERR_ALIGN
    dims, a = _valid_ssm(fused=True)
    a.z = None
    assert _ssm_call(dims, a, fused=True) == nat.M3_ERR_NULL


def test_validation_full_fused():
    lib = nat.load()
    dims = nat.Dims(batch=1, nheads=16, headdim=32, d_state=64, mimo_rank=4, num_rope_angles=16,
                    ngroups=1, d_inner=512, A_floor=1e-4)
    a = nat.FullArgs()
    fake = 0x7000_0000_0000
    for i, f in enumerate(["zx", "dt_bias", "D", "B_norm_w", "C_norm_w", "B_bias", "C_bias",
                           "mimo_x", "mimo_o", "ssm_state", "bx_prev", "angle_state", "y"]):
        setattr(a, f, fake + 4096 * i)
    a.zx_stride_b = 2 * 512 + 2 * 64 * 4 + 3 * 16 + 16 - 1  # one short of d_in_proj
    a.y_stride_b = 512
    assert lib.m3_mimo_full_fused(dims, a, None) == nat.M3_ERR_SHAPE
    a.zx_stride_b += 1
    dims.ngroups = 2
    assert lib.m3_mimo_full_fused(dims, a, None) == nat.M3_ERR_SHAPE
    dims.ngroups = 1
    dims.num_rope_angles = 33
    assert lib.m3_mimo_full_fused(dims, a, None) == nat.M3_ERR_SHAPE
    dims.num_rope_angles = 16
    dims.d_inner = 511
    assert lib.m3_mimo_full_fused(dims, a, None) == nat.M3_ERR_SHAPE
    dims.d_inner = 512
    dims.mimo_rank = 16
    assert lib.m3_mimo_full_fused(dims, a, None) == nat.M3_ERR_RANK
    dims.mimo_rank = 4
    a.param_dtype = 5
    assert lib.m3_mimo_full_fused(dims, a, None) == nat.M3_ERR_DTYPE
    a.param_dtype = nat.M3_F32
    dims.batch = 0  # empty batch: valid, nothing enqueued
    assert lib.m3_mimo_full_fused(dims, a, None) == nat.M3_OK


def test_validation_linear():
    lib = nat.load()
    fake = 0x7000_0000_0000
    ok = (fake, 256, fake + 4096, 256, fake + 8192, 64, 8, 64, 256, None)
    assert lib.m3_linear_f32(None, *ok[1:]) == nat.M3_ERR_NULL
    assert lib.m3_linear_f32(fake, 255, fake + 4096, 256, fake + 8192, 64, 8, 64, 256, None) == nat.M3_ERR_SHAPE
    assert lib.m3_linear_f32(fake, 258, fake + 4096, 258, fake + 8192, 64, 8, 64, 258, None) == nat.M3_ERR_ALIGN
    assert lib.m3_linear_f32(fake + 4, *ok[1:]) == nat.M3_ERR_ALIGN
    assert lib.m3_linear_f32(fake, 256, fake + 4096, 256, fake + 8192, 64, 0, 64, 256, None) == nat.M3_OK


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_no_device_is_reported():
    dims, a = _valid_ssm()
    assert _ssm_call(dims, a) == nat.M3_ERR_DEVICE


def test_status_mapping_to_reference_exceptions():
    with pytest.raises(ValueError):
        nat.check(nat.M3_ERR_RANK, "x")
    with pytest.raises(AssertionError):
        nat.check(nat.M3_ERR_SHAPE, "x")
    with pytest.raises(RuntimeError):
        nat.check(nat.M3_ERR_LAUNCH, "x")
    nat.check(nat.M3_OK, "x")


def _valid_step():
    """A single-launch step call with fake, well-aligned device addresses
    (d_model 256, MIMO rank 4, 16 heads of 32, d_state 64)."""
    lib = nat.load()
    dims = nat.Dims(batch=4, nheads=16, headdim=32, d_state=64, mimo_rank=4, num_rope_angles=16,
                    ngroups=1, d_inner=512, A_floor=1e-4)
    a = nat.StepArgs()
    a.d_model, a.dtype = 256, nat.M3_F32
    fake = 0x7000_0000_0000
    for i, f in enumerate(["u", "in_proj_w", "out_proj_w", "dt_bias", "D", "B_norm_w", "C_norm_w", "B_bias",
                           "C_bias", "mimo_x", "mimo_o", "ssm_state", "bx_prev", "angle_state", "out",
                           "workspace"]):
        setattr(a, f, fake + (1 << 24) * i)
    a.u_stride_b = a.in_proj_stride = a.out_stride_b = 256
    a.out_proj_stride = 512
    a.workspace_bytes = lib.m3_mimo_step_workspace_bytes(dims, 256, nat.M3_F32)
    return lib, dims, a


def test_step_workspace_size_and_range():
    lib, dims, a = _valid_step()
    d_in_proj = 2 * 512 + 2 * 64 * 4 + 3 * 16 + 16
    expect = 256 + -(-4 * d_in_proj * 4 // 256) * 256 + -(-4 * 512 * 4 // 256) * 256
    assert a.workspace_bytes == expect
    assert lib.m3_mimo_step_workspace_bytes(dims, 256, nat.M3_BF16) < expect
    assert lib.m3_mimo_step_workspace_bytes(None, 256, 0) == -nat.M3_ERR_NULL
    assert lib.m3_mimo_step_workspace_bytes(dims, 256, 9) == -nat.M3_ERR_DTYPE
    for field, bad, status in [("nheads", 12, nat.M3_ERR_SHAPE),  # d_inner != H * P
                               ("mimo_rank", 3, nat.M3_ERR_RANK), ("ngroups", 2, nat.M3_ERR_SHAPE)]:
        _, d2, _ = _valid_step()
        setattr(d2, field, bad)
        assert lib.m3_mimo_step_workspace_bytes(d2, 256, 0) == -status, field
    # valid layers outside the kernel's range
    for kw in [dict(nheads=4, d_inner=128), dict(headdim=256, nheads=8, d_inner=2048),
               dict(d_state=256, num_rope_angles=16)]:
        _, d2, _ = _valid_step()
        for k, v in kw.items():
            setattr(d2, k, v)
        assert lib.m3_mimo_step_workspace_bytes(d2, 256, 0) == -nat.M3_ERR_UNSUPPORTED, kw
    assert lib.m3_mimo_step_workspace_bytes(dims, 254, 0) == -nat.M3_ERR_UNSUPPORTED


def test_siso_step_workspace_size_and_range():
    lib = nat.load()
    # the reference's SISO d256 layer: 16 heads x headdim 32, d_state 64
    dims = nat.Dims(batch=4, nheads=16, headdim=32, d_state=64, mimo_rank=1, num_rope_angles=16, ngroups=1,
                    d_inner=512, A_floor=1e-4)
    d_in_proj = 2 * 512 + 2 * 64 + 3 * 16 + 16
    expect = 256 + -(-4 * d_in_proj * 4 // 256) * 256 + -(-4 * 512 * 4 // 256) * 256
    assert lib.m3_siso_step_workspace_bytes(dims, 256, nat.M3_F32) == expect
    # heads need not be a multiple of 8, and d_state 256 / headdim 256 are taken
    for kw in [dict(nheads=4, d_inner=128), dict(headdim=256, nheads=2, d_inner=512),
               dict(d_state=256, num_rope_angles=64)]:
        d2 = nat.Dims(**{**{f: getattr(dims, f) for f, _ in nat.Dims._fields_}, **kw})
        assert lib.m3_siso_step_workspace_bytes(d2, 256, 0) > 0, kw
    d2 = nat.Dims(**{**{f: getattr(dims, f) for f, _ in nat.Dims._fields_}, "mimo_rank": 4})
    assert lib.m3_siso_step_workspace_bytes(d2, 256, 0) == -nat.M3_ERR_SHAPE
    assert lib.m3_siso_step_workspace_bytes(dims, 254, 0) == -nat.M3_ERR_UNSUPPORTED
    assert lib.m3_siso_step_workspace_bytes(None, 256, 0) == -nat.M3_ERR_NULL


def test_step_validation():
    lib, dims, a = _valid_step()
    dims.batch = 0  # a valid call with no rows returns before touching a device
    assert lib.m3_mimo_step(dims, a, None) == nat.M3_OK
    assert lib.m3_mimo_step(None, a, None) == nat.M3_ERR_NULL
    for f in ["u", "in_proj_w", "mimo_o", "angle_state", "out", "workspace"]:
        lib, dims, a = _valid_step()
        setattr(a, f, None)
        assert lib.m3_mimo_step(dims, a, None) == nat.M3_ERR_NULL, f
    lib, dims, a = _valid_step()
    a.workspace_bytes -= 1
    assert lib.m3_mimo_step(dims, a, None) == nat.M3_ERR_SHAPE
    for f, v in [("u_stride_b", 255), ("out_proj_stride", 511), ("out_stride_b", 100)]:
        lib, dims, a = _valid_step()
        setattr(a, f, v)
        assert lib.m3_mimo_step(dims, a, None) == nat.M3_ERR_SHAPE, f
    for f, off in [("u", 4), ("in_proj_w", 8), ("B_bias", 4), ("workspace", 16), ("ssm_state", 8)]:
        lib, dims, a = _valid_step()
        setattr(a, f, getattr(a, f) + off)
        assert lib.m3_mimo_step(dims, a, None) == nat.M3_ERR_ALIGN, f
    lib, dims, a = _valid_step()
    a.in_proj_stride = 258  # >= d_model but not a multiple of 4
    assert lib.m3_mimo_step(dims, a, None) == nat.M3_ERR_ALIGN
    lib, dims, a = _valid_step()
    dims.nheads, dims.d_inner = 4, 128
    assert lib.m3_mimo_step(dims, a, None) == nat.M3_ERR_UNSUPPORTED


def test_static_step_validation_before_any_device_work():
    """The allocation-free step rejects a caller workspace, bad layers and
    batches whose workspace exceeds the library's scratch before it looks
    for a device (status codes only; nothing is enqueued)."""
    text = open(HEADER).read()
    m = re.search(r"#define M3_STEP_STATIC_SCRATCH_BYTES \((\d+) \* (\d+) \* (\d+)\)", text)
    assert m and int(m.group(1)) * int(m.group(2)) * int(m.group(3)) == nat.STEP_STATIC_SCRATCH_BYTES
    lib, dims, a = _valid_step()
    assert lib.m3_mimo_step_static(None, a, None) == nat.M3_ERR_NULL
    assert lib.m3_mimo_step_static(dims, None, None) == nat.M3_ERR_NULL
    assert lib.m3_mimo_step_static(dims, a, None) == nat.M3_ERR_SHAPE  # a caller workspace is not taken
    a.workspace, a.workspace_bytes = None, 0
    dims.mimo_rank = 3
    assert lib.m3_mimo_step_static(dims, a, None) == nat.M3_ERR_RANK
    dims.mimo_rank = 4
    dims.nheads, dims.d_inner = 4, 128
    assert lib.m3_mimo_step_static(dims, a, None) == nat.M3_ERR_UNSUPPORTED
    dims.nheads, dims.d_inner = 16, 512
    dims.batch = 4096  # 4096 rows x 1648 zx columns x 4 bytes > 4 MiB
    assert lib.m3_mimo_step_workspace_bytes(dims, 256, nat.M3_F32) > nat.STEP_STATIC_SCRATCH_BYTES
    assert lib.m3_mimo_step_static(dims, a, None) == nat.M3_ERR_SCRATCH
    assert "static scratch" in nat.status_string(nat.M3_ERR_SCRATCH)
