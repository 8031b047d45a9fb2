"""GPU parity of the streamed MIMO full-step kernel (mimo_stream_kernel).

The fused MIMO entry point takes the streamed kernel whenever every piece of
a batch row can be bulk-copied (8 heads per CTA, headdim 32/64/128, d_state
36..256, 16-byte aligned sections).  These cases are chosen to land on it:
state widths 64/96/128/256 (one and two vectors per lane, padded lanes),
headdims 32/64/128, every rank, rope_fraction 1.0, fp32 and bf16, batches
that give one or many rows per CTA (one-row and two-row passes, an odd
row count whose last pass has one live row), more than one 32-row chunk of the
head-scalar table, and accumulated angles far from zero (both the reduced
and the full-range sin/cos).  Oracle tolerance 1e-4 in fp32.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mamba3_oracle as orc
from test_full_fused_gpu import TOL, _compare, _kernel, _random_state, _t

pytestmark = pytest.mark.gpu

LAYERS = [
    # layer kwargs (8 heads or more, stream-eligible), batch
    (dict(d_model=512, d_state=64, headdim=64), 5),       # D 64: 2 floats per lane
    (dict(d_model=512, d_state=128, headdim=64), 37),     # D 128: 4 floats per lane
    (dict(d_model=1024, d_state=256, headdim=128), 3),    # D 256: 2 vectors per lane, headdim 128
    (dict(d_model=128, d_state=96, headdim=32), 300),     # D 96 (padded lanes), headdim 32, rows per CTA > 1
    (dict(d_model=512, d_state=128, headdim=64, rope_fraction=1.0), 4),  # every pair rotates
    (dict(d_model=256, d_state=128, headdim=64), 601),    # 3 rows per CTA, last CTA 1: two-row passes with a tail
    (dict(d_model=512, d_state=128, headdim=64, rope_fraction=1.0), 900),  # two-row passes, every pair rotates
]


@pytest.mark.parametrize("R", [1, 2, 4, 8])
@pytest.mark.parametrize("kw,batch", LAYERS, ids=lambda v: str(v))
def test_stream_matches_oracle(kw, batch, R):
    dims = orc.layer_dims(**kw, is_mimo=True, mimo_rank=R)
    assert dims["nheads"] % 8 == 0
    _compare(dims, orc.synthetic_params(dims, 30 + R), batch, steps=3, seed=31 + R)


@pytest.mark.parametrize("R", [2, 8])
def test_stream_bf16(R):
    dims = orc.layer_dims(d_model=512, d_state=128, headdim=64, is_mimo=True, mimo_rank=R)
    _compare(dims, orc.synthetic_params(dims, 40 + R, bf16=True), 19, steps=3, seed=41, zx_bf16=True)


def test_stream_many_rows_per_cta():
    """20000 rows (about 68 per CTA: three chunks of the head-scalar table)
    that repeat 8 distinct rows give those rows' results, and the 8 rows
    match the oracle."""
    dims = orc.layer_dims(d_model=256, d_state=128, headdim=64, is_mimo=True, mimo_rank=4)
    assert dims["nheads"] == 8
    params = orc.synthetic_params(dims, 50)
    rng = np.random.default_rng(51)
    small = _random_state(dims, 8, rng)
    zx8 = (rng.standard_normal((8, dims["d_in_proj"])) * 0.6).astype(np.float32)
    rep = 2500
    big = {k: _t(np.tile(v, (rep,) + (1,) * (v.ndim - 1))) for k, v in small.items()}
    yb = _kernel(dims, params, _t(np.tile(zx8, (rep, 1))), big)
    ye, a, h, bx = orc.ssm_from_zx(zx8, params, dims, small["angle_state"], small["ssm_state"], small["bx_prev"])
    yb = yb.cpu().numpy().reshape(rep, 8, *ye.shape[1:])
    np.testing.assert_allclose(yb[0], ye, **TOL)
    assert (yb == yb[:1]).all(), "repeated rows differ"
    for name, want in (("angle_state", a), ("ssm_state", h), ("bx_prev", bx)):
        got = big[name].cpu().numpy().reshape(rep, 8, *want.shape[1:])
        np.testing.assert_allclose(got[0], want, **TOL, err_msg=name)
        assert (got == got[:1]).all(), name


def test_stream_large_angles():
    """Accumulated angles of magnitude up to 3e5 (no increment this step, so
    the angles stay exact): the rotation uses the reduced sin/cos below 2^17
    and the full-range one above."""
    dims = orc.layer_dims(d_model=512, d_state=128, headdim=64, is_mimo=True, mimo_rank=4)
    params = orc.synthetic_params(dims, 60)
    rng = np.random.default_rng(61)
    B = 16
    st_np = _random_state(dims, B, rng)
    mag = 10.0 ** rng.uniform(2, np.log10(3e5), st_np["angle_state"].shape)
    st_np["angle_state"] = (np.sign(rng.standard_normal(mag.shape)) * mag).astype(np.float32)
    zx = (rng.standard_normal((B, dims["d_in_proj"])) * 0.6).astype(np.float32)
    H, A = dims["nheads"], dims["num_rope_angles"]
    so = 2 * dims["d_inner"] + 2 * dims["d_state"] * dims["mimo_rank"]
    zx[:, so + 3 * H:so + 3 * H + A] = 0.0
    st = {k: _t(v) for k, v in st_np.items()}
    y = _kernel(dims, params, _t(zx), st)
    ye, a, h, bx = orc.ssm_from_zx(zx, params, dims, st_np["angle_state"], st_np["ssm_state"], st_np["bx_prev"])
    np.testing.assert_array_equal(st["angle_state"].cpu().numpy(), a)
    np.testing.assert_allclose(y.cpu().numpy(), ye, **TOL)
    np.testing.assert_allclose(st["ssm_state"].cpu().numpy(), h, **TOL)
    np.testing.assert_allclose(st["bx_prev"].cpu().numpy(), bx, **TOL)

