"""Pin the numpy oracle to the reference (CPU only).

The fixtures under tests/golden were produced by running the reference's own
PyTorch decode path (see tests/golden/make_golden.py).  Here the oracle is
re-run on the same seeded inputs and must reproduce them; the known-answer
and closed-form checks mirror the reference tests
(src/tests/test_trapezoidal.py, src/tests/test_siso.py:135-195,
src/tests/test_mimo.py:149-216).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_names, layer_kwargs, load_golden
from oracle import mamba3_oracle as orc


def _run_layer_oracle(g):
    m = g["meta"]
    dims = orc.layer_dims(**layer_kwargs(m["layer"]))
    params = orc.synthetic_params(dims, m["param_seed"], bf16=m["bf16"])
    u = orc.synthetic_inputs(dims, m["batch"], m["steps"], m["input_seed"], bf16=m["bf16"])
    st = orc.init_state(dims, m["batch"])
    outs = []
    for t in range(m["steps"]):
        o, st = orc.decode_step(u[t], params, dims, st, bf16=m["bf16"])
        outs.append(o)
    return dims, params, np.stack(outs), st


@pytest.mark.parametrize("name", golden_names("layer"))
def test_layer_oracle_matches_reference(name):
    g = load_golden(name)
    dims, params, out, st = _run_layer_oracle(g)
    if g["meta"]["bf16"]:
        # bf16 outputs: allow a couple of bf16 ulps (the in_proj rounding can
        # land on the other side of a bf16 boundary when the fp32 sums differ
        # in their last bit)
        np.testing.assert_allclose(out, g["out"], rtol=2e-2, atol=2e-3)
        np.testing.assert_allclose(st["angle_state"], g["angle_state"], rtol=1e-3, atol=1e-4)
        h = st["ssm_state"].reshape(st["ssm_state"].shape[0], dims["nheads"], -1)
        np.testing.assert_allclose(h.sum(-1), g["ssm_sum"], rtol=1e-2, atol=1e-3)
    else:
        np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(st["angle_state"], g["angle_state"], rtol=1e-5, atol=1e-6)
        h = st["ssm_state"].reshape(st["ssm_state"].shape[0], dims["nheads"], -1)
        np.testing.assert_allclose(h.sum(-1), g["ssm_sum"], rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose((h.astype(np.float64) ** 2).sum(-1), g["ssm_sumsq"], rtol=1e-4)
        if "ssm_state" in g:
            np.testing.assert_allclose(st["ssm_state"], g["ssm_state"], rtol=1e-4, atol=1e-5)
            np.testing.assert_allclose(st["bx_prev"], g["bx_prev"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("name", [n for n in golden_names("layer") if load_golden(n)["meta"]["bf16"]])
def test_bf16_oracle_post_gemm_matches_reference(name):
    """Feeding the reference's own bf16 in_proj outputs removes the GEMM
    rounding from the comparison: the rest of the step must agree tightly."""
    g = load_golden(name)
    m = g["meta"]
    dims = orc.layer_dims(**layer_kwargs(m["layer"]))
    params = orc.synthetic_params(dims, m["param_seed"], bf16=True)
    st = orc.init_state(dims, m["batch"])
    for t in range(m["steps"]):
        _, a, h, bx = orc.ssm_from_zx(g["zx"][t], params, dims, st["angle_state"],
                                      st["ssm_state"], st["bx_prev"])
        st = {"angle_state": a, "ssm_state": h, "bx_prev": bx}
    np.testing.assert_allclose(st["angle_state"], g["angle_state"], rtol=1e-5, atol=1e-6)
    hs = st["ssm_state"].reshape(m["batch"], dims["nheads"], -1)
    np.testing.assert_allclose(hs.sum(-1), g["ssm_sum"], rtol=1e-4, atol=1e-4)
    if "ssm_state" in g:
        np.testing.assert_allclose(st["ssm_state"], g["ssm_state"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("name", golden_names("ssm"))
def test_ssm_oracle_matches_reference(name):
    g = load_golden(name)
    m = g["meta"]
    d = orc.ssm_kernel_inputs(m["ssm_kind"], m["B"], m["H"], m["P"], m["D"], m["R"],
                              m["seed"], m["trap_value"])
    if m["ssm_kind"] == "siso":
        y, h, bx = orc.siso_decode(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"],
                                   d["trap"], d["D_skip"], d["h"], d["bx_prev"])
    else:
        y, h, bx = orc.mimo_decode(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"],
                                   d["trap"], d["D_skip"], d["mimo_x"], d["mimo_o"],
                                   d["h"], d["bx_prev"])
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(h.sum(-1), g["h_sum"], rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(bx.sum(-1), g["bx_sum"], rtol=1e-5, atol=1e-4)
    if "h" in g:
        np.testing.assert_allclose(h, g["h"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(bx, g["bx"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", golden_names("stack"))
def test_stack_oracle_matches_reference(name):
    g = load_golden(name)
    m = g["meta"]
    dims = orc.layer_dims(**layer_kwargs(m["layer"]))
    rng = np.random.default_rng(m["seed"])
    layers = []
    for l in range(m["layers"]):
        params = orc.synthetic_params(dims, m["seed"] + 1 + l, bf16=m["bf16"])
        w = (1.0 + 0.2 * rng.standard_normal(dims["d_model"])).astype(np.float32)
        layers.append((params, w, orc.init_state(dims, m["batch"])))
    u = orc.synthetic_inputs(dims, m["batch"], m["steps"], m["seed"] + 100, bf16=m["bf16"])
    outs = []
    for t in range(m["steps"]):
        x = u[t]
        for l, (params, w, st) in enumerate(layers):
            x, st = orc.residual_block_step(x, w, params, dims, st, bf16=m["bf16"])
            layers[l] = (params, w, st)
        outs.append(x)
    np.testing.assert_allclose(np.stack(outs), g["out"], rtol=2e-2, atol=2e-2)


# --------------------------------------------------------------------------
# known answers and closed forms (reference test suite)
# --------------------------------------------------------------------------

def test_rope_known_answer():
    """src/tests/test_trapezoidal.py:101-117: [1,0,0,1] rotated by [0, pi/2]."""
    out = orc.apply_rope(np.array([1.0, 0.0, 0.0, 1.0], np.float32),
                         np.array([0.0, np.pi / 2], np.float32))
    np.testing.assert_allclose(out, [1.0, 0.0, -1.0, 0.0], atol=1e-6)


def test_rope_zero_angle_identity():
    x = np.random.default_rng(0).standard_normal((4, 8)).astype(np.float32)
    np.testing.assert_allclose(orc.apply_rope(x, np.zeros((4, 4), np.float32)), x, atol=1e-6)


def test_trap_gate_interpolation():
    """src/tests/test_trapezoidal.py:17-58."""
    bx = np.array([1.0, 2.0], np.float32)
    prev = np.array([3.0, 4.0], np.float32)
    np.testing.assert_allclose(orc.trapezoidal_blend(bx, prev, np.float32(0.0)), bx, atol=1e-6)
    np.testing.assert_allclose(orc.trapezoidal_blend(bx, prev, np.float32(1.0)), 0.5 * (bx + prev), atol=1e-6)
    np.testing.assert_allclose(orc.trapezoidal_blend(bx, prev, np.float32(0.5)),
                               0.5 * bx + 0.25 * (bx + prev), atol=1e-6)


@pytest.mark.parametrize("kind", ["siso", "mimo"])
@pytest.mark.parametrize("trap_value", [0.0, 1.0])
def test_trap_closed_forms(kind, trap_value):
    """trap=0 is Euler, trap=1 the trapezoid average (src/tests/test_siso.py:135-195,
    src/tests/test_mimo.py:149-216), tolerance 1e-5."""
    d = orc.ssm_kernel_inputs(kind, 1, 2, 8, 16, 2, 7, trap_value)
    h0 = np.zeros_like(d["h"])
    if kind == "siso":
        _, h, _ = orc.siso_decode(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"], d["trap"],
                                  d["D_skip"], h0, d["bx_prev"])
        bx = d["x"][..., :, None] * d["B_proj"][..., None, :]
        dt = d["DT"][..., None, None]
    else:
        _, h, _ = orc.mimo_decode(d["x"], d["B_proj"], d["C_proj"], d["ADT"], d["DT"], d["trap"],
                                  d["D_skip"], d["mimo_x"], d["mimo_o"], h0, d["bx_prev"])
        xr = np.einsum("bhp,hrp->bhr", d["x"], d["mimo_x"])
        bx = np.einsum("bhr,brhd->bhd", xr, d["B_proj"])
        dt = d["DT"][..., None]
    expect = dt * (bx if trap_value == 0.0 else 0.5 * (bx + d["bx_prev"]))
    np.testing.assert_allclose(h, expect, atol=1e-5)


def test_A_floor_quirk():
    """A = -(softplus(dd_A).clamp(max=-A_floor)) is +A_floor for every input
    (src/models/mamba3.py:196)."""
    dims = orc.layer_dims(d_model=64, d_state=16, headdim=16)
    params = orc.synthetic_params(dims, 0)
    zx = np.random.default_rng(1).standard_normal((3, dims["d_in_proj"])).astype(np.float32) * 5
    _, _, _, _, ADT, DT, _, _ = orc.compute_params(zx, params, dims)
    np.testing.assert_allclose(ADT, np.float32(1e-4) * DT, rtol=1e-6)


def test_bf16_rounding_matches_torch():
    import torch
    x = np.random.default_rng(3).standard_normal(4096).astype(np.float32) * 100
    x[:4] = [np.inf, -np.inf, np.nan, 0.0]
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(orc.round_bf16(x), ref)
