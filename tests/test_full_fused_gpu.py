"""GPU parity of the full-step fused kernels (``mamba3_{siso,mimo}_full_fused_triton``)
against the oracle's restatement of the reference step between in_proj and
out_proj (src/models/mamba3.py:321-349), on identical in_proj outputs.

Covers SISO and MIMO R in {1, 2, 4, 8}, d_state 16..256 (powers of two and
not), odd headdims, rope_fraction 1.0, non-default A_floor, fp32 and bf16
in_proj outputs / parameters, chained steps from a non-zero state, the
reference fixtures' own bf16 in_proj outputs, and batch independence at a
large batch.  fp32 tolerance 1e-4 (build target 1e-3).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, layer_kwargs, load_golden
from oracle import mamba3_oracle as orc
from src.kernels.fused_full_decode import mamba3_mimo_full_fused_triton, mamba3_siso_full_fused_triton

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-4, atol=1e-4)


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dtype)


def _kernel(dims, params, zx, st, pdtype=torch.float32):
    """Run one fused step on GPU tensors ``st`` (updated in place)."""
    H, R = dims["nheads"], dims["mimo_rank"]
    p = {k: _t(v, pdtype) for k, v in params.items() if k not in ("in_proj_weight", "out_proj_weight")}
    kw = dict(d_inner=dims["d_inner"], d_state=dims["d_state"], ngroups=1, mimo_rank=R, nheads=H,
              headdim=dims["headdim"], split_tensor_size=dims["split"],
              num_rope_angles=dims["num_rope_angles"], A_floor=dims["A_floor"])
    if dims["is_mimo"]:
        y, h, bx, a = mamba3_mimo_full_fused_triton(
            zx, p["dt_bias"], p["D"], p["B_norm_weight"], p["C_norm_weight"], p["B_bias"], p["C_bias"],
            p["mimo_x"], p["mimo_o"], st["ssm_state"], st["bx_prev"], st["angle_state"], **kw)
    else:
        y, h, bx, a = mamba3_siso_full_fused_triton(
            zx, p["dt_bias"], p["D"], p["B_norm_weight"], p["C_norm_weight"], p["B_bias"][:, 0],
            p["C_bias"][:, 0], st["ssm_state"], st["bx_prev"], st["angle_state"], **kw)
    assert h is st["ssm_state"] and bx is st["bx_prev"] and a is st["angle_state"]
    assert y.dtype == torch.float32 and y.shape == (zx.shape[0], H, dims["headdim"])
    return y


def _random_state(dims, batch, rng):
    st = orc.init_state(dims, batch)
    return {k: (rng.standard_normal(v.shape) * 0.5).astype(np.float32) for k, v in st.items()}


def _compare(dims, params, batch, steps, seed, zx_bf16=False, tol=TOL):
    rng = np.random.default_rng(seed)
    st_np = _random_state(dims, batch, rng)
    st = {k: _t(v) for k, v in st_np.items()}
    pdtype = torch.bfloat16 if zx_bf16 else torch.float32
    for _ in range(steps):
        zx = (rng.standard_normal((batch, dims["d_in_proj"])) * 0.6).astype(np.float32)
        if zx_bf16:
            zx = orc.round_bf16(zx)
        y = _kernel(dims, params, _t(zx, pdtype), st, pdtype)
        ye, a, h, bx = orc.ssm_from_zx(zx, params, dims, st_np["angle_state"], st_np["ssm_state"],
                                       st_np["bx_prev"])
        st_np = {"angle_state": a, "ssm_state": h, "bx_prev": bx}
        np.testing.assert_allclose(y.cpu().numpy(), ye, **tol)
    for k in st_np:
        np.testing.assert_allclose(st[k].cpu().numpy(), st_np[k], **tol, err_msg=k)


LAYERS = [
    # (layer kwargs, batch)
    (dict(d_model=256, d_state=64, headdim=32), 2),                          # SISO d256
    (dict(d_model=64, d_state=16, headdim=16), 3),
    (dict(d_model=64, d_state=32, headdim=16, rope_fraction=1.0, A_floor=1e-3), 2),
    (dict(d_model=128, d_state=128, headdim=64), 2),
    (dict(d_model=64, d_state=256, headdim=32), 1),
    (dict(d_model=96, d_state=48, headdim=24), 2),                           # non-power-of-two D, P
    (dict(d_model=40, d_state=96, headdim=20, rope_fraction=1.0), 2),
    (dict(d_model=48, d_state=16, headdim=32), 3),                           # 3 heads: unaligned sections
]


@pytest.mark.parametrize("kw,batch", LAYERS)
def test_siso_full_fused(kw, batch):
    dims = orc.layer_dims(**kw)
    _compare(dims, orc.synthetic_params(dims, 1), batch, steps=4, seed=2)


@pytest.mark.parametrize("R", [1, 2, 4, 8])
@pytest.mark.parametrize("kw,batch", LAYERS)
def test_mimo_full_fused(kw, batch, R):
    dims = orc.layer_dims(**kw, is_mimo=True, mimo_rank=R)
    _compare(dims, orc.synthetic_params(dims, 3 + R), batch, steps=4, seed=4 + R)


@pytest.mark.parametrize("mimo", [False, True])
def test_bf16_in_proj_output_and_params(mimo):
    dims = orc.layer_dims(d_model=128, d_state=64, headdim=32, is_mimo=mimo, mimo_rank=4)
    _compare(dims, orc.synthetic_params(dims, 5, bf16=True), 3, steps=3, seed=6, zx_bf16=True)


@pytest.mark.parametrize("mimo", [False, True])
def test_mixed_dtypes_bf16_zx_f32_params(mimo):
    """bf16 in_proj output with fp32 parameters (the generic MIMO path)."""
    dims = orc.layer_dims(d_model=128, d_state=64, headdim=32, is_mimo=mimo, mimo_rank=2)
    params = orc.synthetic_params(dims, 21)
    rng = np.random.default_rng(22)
    st_np = _random_state(dims, 3, rng)
    st = {k: _t(v) for k, v in st_np.items()}
    zx = orc.round_bf16((rng.standard_normal((3, dims["d_in_proj"])) * 0.6).astype(np.float32))
    y = _kernel(dims, params, _t(zx, torch.bfloat16), st, torch.float32)
    ye, a, h, bx = orc.ssm_from_zx(zx, params, dims, st_np["angle_state"], st_np["ssm_state"],
                                   st_np["bx_prev"])
    np.testing.assert_allclose(y.cpu().numpy(), ye, **TOL)
    np.testing.assert_allclose(st["ssm_state"].cpu().numpy(), h, **TOL)


def test_bounded_wait_reports_timeout():
    """A wait on a barrier nothing completes gives up and sets the device
    error word instead of hanging; the context stays usable."""
    from src import _native as nat
    lib = nat.load()
    assert nat.device_error(reset=True) == 0
    assert lib.m3_selftest_wait_timeout(torch.cuda.current_stream().cuda_stream) == nat.M3_OK
    torch.cuda.synchronize()
    assert nat.device_error(reset=True) == nat.M3_DEVERR_TIMEOUT
    assert nat.device_error() == 0
    x = torch.ones(4, device="cuda")
    assert (x + 1).sum().item() == 8.0


@pytest.mark.parametrize("name", [n for n in golden_names("layer") if load_golden(n)["meta"]["bf16"]])
def test_reference_bf16_zx_fixtures(name):
    """Feed the reference's own bf16 in_proj outputs; the final state must
    match the reference's (summaries; full state where stored)."""
    g = load_golden(name)
    m = g["meta"]
    dims = orc.layer_dims(**layer_kwargs(m["layer"]))
    params = orc.synthetic_params(dims, m["param_seed"], bf16=True)
    st = {k: _t(v) for k, v in orc.init_state(dims, m["batch"]).items()}
    for t in range(m["steps"]):
        _kernel(dims, params, _t(g["zx"][t], torch.bfloat16), st, torch.bfloat16)
    np.testing.assert_allclose(st["angle_state"].cpu().numpy(), g["angle_state"], **TOL)
    h = st["ssm_state"].cpu().numpy().reshape(m["batch"], dims["nheads"], -1)
    np.testing.assert_allclose(h.sum(-1), g["ssm_sum"], rtol=1e-4, atol=1e-3)
    if "ssm_state" in g:
        np.testing.assert_allclose(st["ssm_state"].cpu().numpy(), g["ssm_state"], **TOL)


@pytest.mark.parametrize("mimo", [False, True])
def test_large_batch_rows_are_independent(mimo):
    """4096 rows that repeat 8 distinct rows must give the 8 rows' results."""
    dims = orc.layer_dims(d_model=256, d_state=64, headdim=32, is_mimo=mimo, mimo_rank=4)
    params = orc.synthetic_params(dims, 9)
    rng = np.random.default_rng(10)
    small = _random_state(dims, 8, rng)
    zx8 = (rng.standard_normal((8, dims["d_in_proj"])) * 0.6).astype(np.float32)
    rep = 512
    big = {k: _t(np.tile(v, (rep,) + (1,) * (v.ndim - 1))) for k, v in small.items()}
    sm = {k: _t(v) for k, v in small.items()}
    yb = _kernel(dims, params, _t(np.tile(zx8, (rep, 1))), big)
    ys = _kernel(dims, params, _t(zx8), sm)
    ys_rep = ys.repeat(rep, 1, 1)
    torch.testing.assert_close(yb, ys_rep, rtol=0, atol=0)
    for k in big:
        torch.testing.assert_close(big[k], sm[k].repeat((rep,) + (1,) * (sm[k].dim() - 1)), rtol=0, atol=0)


def test_zero_batch_and_errors():
    dims = orc.layer_dims(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2)
    params = orc.synthetic_params(dims, 0)
    st = {k: _t(v) for k, v in orc.init_state(dims, 0).items()}
    y = _kernel(dims, params, torch.zeros(0, dims["d_in_proj"], device="cuda"), st)
    assert y.shape == (0, dims["nheads"], dims["headdim"])
    st = {k: _t(v) for k, v in orc.init_state(dims, 2).items()}
    with pytest.raises(AssertionError):  # wrong in_proj width
        _kernel(dims, params, torch.zeros(2, dims["d_in_proj"] + 1, device="cuda"), st)
    d3 = dict(dims, mimo_rank=3)
    with pytest.raises((ValueError, AssertionError)):
        _kernel(d3, params, torch.zeros(2, dims["d_in_proj"], device="cuda"), st)
