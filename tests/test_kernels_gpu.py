"""GPU parity of the state-update-only kernels (the ``use_triton`` /
``use_triton_fused`` entry points) against the oracle and the reference
fixtures.  Cases mirror the reference's src/tests/test_siso.py and
src/tests/test_mimo.py (shapes, seeds, closed forms) plus strided views,
bf16 activations, odd sizes and error mapping.

Tolerance: 1e-4 absolute/relative for a single step in fp32 (the reference
tests use 1e-2; the build target is 1e-3); the closed forms use 1e-5 as in
the reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import mamba3_oracle as orc
from src.kernels.mimo_decode import mamba3_mimo_decode_triton
from src.kernels.mimo_decode_fused import mamba3_mimo_decode_fused_triton
from src.kernels.siso_decode import mamba3_siso_decode_triton
from src.kernels.siso_decode_fused import mamba3_siso_decode_fused_triton

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-4, atol=1e-4)


def _cuda(d):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in d.items()}


def _run(kind, t, gated=False):
    h, bx = t["h"].clone(), t["bx_prev"].clone()
    if kind == "siso":
        if gated:
            y, h2, bx2 = mamba3_siso_decode_fused_triton(t["x"], t["B_proj"], t["C_proj"], t["ADT"],
                                                         t["DT"], t["trap"], t["D_skip"], t["z"], h, bx)
        else:
            y, h2, bx2 = mamba3_siso_decode_triton(t["x"], t["B_proj"], t["C_proj"], t["ADT"], t["DT"],
                                                   t["trap"], t["D_skip"], h, bx)
    else:
        if gated:
            y, h2, bx2 = mamba3_mimo_decode_fused_triton(t["x"], t["B_proj"], t["C_proj"], t["ADT"],
                                                         t["DT"], t["trap"], t["D_skip"], t["mimo_x"],
                                                         t["mimo_o"], t["z"], h, bx)
        else:
            y, h2, bx2 = mamba3_mimo_decode_triton(t["x"], t["B_proj"], t["C_proj"], t["ADT"], t["DT"],
                                                   t["trap"], t["D_skip"], t["mimo_x"], t["mimo_o"], h, bx)
    assert h2 is h and bx2 is bx  # updated in place and returned
    return y, h, bx


def _oracle(kind, d, gated=False):
    if kind == "siso":
        y, h, bx = orc.siso_decode(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"], d["trap"],
                                   d["D_skip"], d["h"], d["bx_prev"])
    else:
        y, h, bx = orc.mimo_decode(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"], d["trap"],
                                   d["D_skip"], d["mimo_x"], d["mimo_o"], d["h"], d["bx_prev"])
    if gated:
        y = (y * orc.silu(d["z"])).astype(np.float32)
    return y, h, bx


def _check(kind, d, gated=False, tol=TOL):
    y, h, bx = _run(kind, _cuda(d), gated)
    ye, he, bxe = _oracle(kind, d, gated)
    np.testing.assert_allclose(y.float().cpu().numpy(), ye, **tol)
    np.testing.assert_allclose(h.cpu().numpy(), he, **tol)
    np.testing.assert_allclose(bx.cpu().numpy(), bxe, **tol)


@pytest.mark.parametrize("name", golden_names("ssm"))
def test_against_reference_fixtures(name):
    g = load_golden(name)
    m = g["meta"]
    d = orc.ssm_kernel_inputs(m["ssm_kind"], m["B"], m["H"], m["P"], m["D"], m["R"], m["seed"],
                              m["trap_value"])
    y, h, bx = _run(m["ssm_kind"], _cuda(d))
    np.testing.assert_allclose(y.cpu().numpy(), g["y"], **TOL)
    np.testing.assert_allclose(h.cpu().numpy().sum(-1), g["h_sum"], rtol=1e-4, atol=1e-3)
    if "h" in g:
        np.testing.assert_allclose(h.cpu().numpy(), g["h"], **TOL)
        np.testing.assert_allclose(bx.cpu().numpy(), g["bx"], **TOL)


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("P,D", [(16, 64), (32, 128), (64, 64), (8, 16), (24, 32), (7, 48), (64, 256),
                                 (100, 96), (1, 4)])
def test_siso_sizes(P, D, gated):
    _check("siso", orc.ssm_kernel_inputs("siso", 2, 4, P, D, 1, 42 + P + D), gated)


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("R", [1, 2, 4, 8])
@pytest.mark.parametrize("P,D", [(16, 64), (64, 128), (32, 16), (24, 48), (5, 256), (70, 32)])
def test_mimo_ranks_and_sizes(R, P, D, gated):
    _check("mimo", orc.ssm_kernel_inputs("mimo", 3, 5, P, D, R, 7 * R + P + D), gated)


@pytest.mark.parametrize("kind", ["siso", "mimo"])
@pytest.mark.parametrize("trap_value", [0.0, 1.0])
def test_trap_closed_forms(kind, trap_value):
    """trap=0 -> Euler, trap=1 -> trapezoid (src/tests/test_siso.py:135-195,
    src/tests/test_mimo.py:149-216), at 1e-5."""
    d = orc.ssm_kernel_inputs(kind, 1, 2, 8, 16, 2, 42, trap_value)
    d["h"] = np.zeros_like(d["h"])
    _, h, _ = _run(kind, _cuda(d))
    if kind == "siso":
        bx = d["x"][..., :, None] * d["B_proj"][..., None, :]
        dt = d["DT"][..., None, None]
    else:
        xr = np.einsum("bhp,hrp->bhr", d["x"], d["mimo_x"])
        bx = np.einsum("bhr,brhd->bhd", xr, d["B_proj"])
        dt = d["DT"][..., None]
    expect = dt * (bx if trap_value == 0.0 else 0.5 * (bx + d["bx_prev"]))
    np.testing.assert_allclose(h.cpu().numpy(), expect, atol=1e-5, rtol=0)


def test_strided_views_like_the_partial_backends():
    """x, z, B, C, ADT... as non-contiguous views of one projection, the way
    the PyTorch prep of the partially fused backends produces them."""
    torch.manual_seed(0)
    Bsz, H, P, D, R = 3, 4, 16, 32, 2
    big = torch.randn(Bsz, 2 * H * P + 2 * R * H * D + 3 * H, device="cuda")
    z, x, Bp, Cp, adt, dt, tr = torch.split(big, [H * P, H * P, R * H * D, R * H * D, H, H, H], dim=-1)
    x, z = x.view(Bsz, H, P), z.view(Bsz, H, P)
    Bp, Cp = Bp.reshape(Bsz, R, H, D), Cp.reshape(Bsz, R, H, D)
    adt, dt, tr = -adt.abs() * 0.1, dt.abs() * 0.1, torch.sigmoid(tr)
    Dsk = torch.randn(H, device="cuda")
    mx = torch.randn(R, H, P, device="cuda").transpose(0, 1)  # (H, R, P), non-contiguous
    mo = torch.randn(H, R, P, device="cuda")
    h = torch.randn(Bsz, H, D, device="cuda")
    bx = torch.randn(Bsz, H, D, device="cuda")
    assert not x.is_contiguous() and not mx.is_contiguous()
    d = {k: v.cpu().numpy() for k, v in dict(x=x, B_proj=Bp, C_proj=Cp, ADT=adt, DT=dt, trap=tr,
                                               D_skip=Dsk, mimo_x=mx, mimo_o=mo, h=h, bx_prev=bx,
                                               z=z).items()}
    y, h2, bx2 = mamba3_mimo_decode_fused_triton(x, Bp, Cp, adt, dt, tr, Dsk, mx, mo, z, h, bx)
    ye, he, bxe = _oracle("mimo", d, gated=True)
    np.testing.assert_allclose(y.cpu().numpy(), ye, **TOL)
    np.testing.assert_allclose(h.cpu().numpy(), he, **TOL)
    # SISO with rank-0 slices (B_proj[:, 0] of a (B, 1, H, D) view)
    hs = torch.randn(Bsz, H, P, D, device="cuda")
    bs = torch.randn(Bsz, H, P, D, device="cuda")
    d.update(h=hs.cpu().numpy(), bx_prev=bs.cpu().numpy(), B_proj=d["B_proj"][:, 0],
             C_proj=d["C_proj"][:, 0])
    y, _, _ = mamba3_siso_decode_triton(x, Bp[:, 0], Cp[:, 0], adt, dt, tr, Dsk, hs, bs)
    ye, he, _ = _oracle("siso", d)
    np.testing.assert_allclose(y.cpu().numpy(), ye, **TOL)
    np.testing.assert_allclose(hs.cpu().numpy(), he, **TOL)


def test_bf16_activations():
    """bf16 x and z (as produced by a bf16 in_proj): y comes back bf16,
    computed in fp32 from the exact bf16 values."""
    d = orc.ssm_kernel_inputs("siso", 2, 4, 16, 64, 1, 3)
    d["x"] = orc.round_bf16(d["x"])
    d["z"] = orc.round_bf16(d["z"])
    t = _cuda(d)
    t["x"], t["z"] = t["x"].bfloat16(), t["z"].bfloat16()
    y, h, _ = _run("siso", t, gated=True)
    assert y.dtype == torch.bfloat16
    ye, he, _ = _oracle("siso", d, gated=True)
    np.testing.assert_allclose(y.float().cpu().numpy(), orc.round_bf16(ye), rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(h.cpu().numpy(), he, **TOL)


def test_empty_batch():
    d = _cuda(orc.ssm_kernel_inputs("mimo", 1, 2, 8, 16, 2, 0))
    for k in ("x", "B_proj", "C_proj", "ADT", "DT", "trap", "h", "bx_prev"):
        d[k] = d[k][:0]
    y, h, bx = _run("mimo", d)
    assert y.shape == (0, 2, 8)


def test_error_mapping():
    d = _cuda(orc.ssm_kernel_inputs("mimo", 1, 2, 8, 16, 2, 0))
    bad = {k: v for k, v in d.items()}
    bad["B_proj"] = torch.randn(1, 3, 2, 16, device="cuda")
    bad["C_proj"] = torch.randn(1, 3, 2, 16, device="cuda")
    bad["mimo_x"] = torch.randn(2, 3, 8, device="cuda")
    bad["mimo_o"] = torch.randn(2, 3, 8, device="cuda")
    with pytest.raises(ValueError):
        _run("mimo", bad)
    with pytest.raises(AssertionError):  # non-contiguous state
        h = torch.randn(1, 16, 2, device="cuda").transpose(1, 2)
        mamba3_mimo_decode_triton(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"], d["trap"],
                                  d["D_skip"], d["mimo_x"], d["mimo_o"], h, d["bx_prev"].clone())
    with pytest.raises(AssertionError):  # state on the host
        mamba3_mimo_decode_triton(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"], d["trap"],
                                  d["D_skip"], d["mimo_x"], d["mimo_o"], d["h"].cpu(), d["bx_prev"])
    with pytest.raises(AssertionError):  # unsupported d_state (not a multiple of 4)
        s = _cuda(orc.ssm_kernel_inputs("siso", 1, 2, 8, 6, 1, 0))
        _run("siso", s)


def test_repeated_steps_accumulate_like_the_oracle():
    """Ten chained steps on the same tensors (state carried in place)."""
    rng = np.random.default_rng(5)
    d = orc.ssm_kernel_inputs("siso", 2, 3, 16, 32, 1, 11)
    t = _cuda(d)
    h, bx = t["h"].clone(), t["bx_prev"].clone()
    he, bxe = d["h"], d["bx_prev"]
    for _ in range(10):
        x = rng.standard_normal(d["x"].shape).astype(np.float32)
        y, _, _ = mamba3_siso_decode_triton(torch.from_numpy(x).cuda(), t["B_proj"], t["C_proj"], t["ADT"],
                                            t["DT"], t["trap"], t["D_skip"], h, bx)
        ye, he, bxe = orc.siso_decode(x, d["B_proj"], d["C_proj"], d["ADT"], d["DT"], d["trap"],
                                      d["D_skip"], he, bxe)
    np.testing.assert_allclose(y.cpu().numpy(), ye, **TOL)
    np.testing.assert_allclose(h.cpu().numpy(), he, **TOL)
