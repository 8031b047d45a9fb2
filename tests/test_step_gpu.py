"""GPU tests of the single-launch decode step (m3_mimo_step, m3_siso_step).

The kernel computes in_proj, the full-step update and out_proj in one
cooperative launch.  It is checked against the oracle (fp32, 1e-4) and
against the three-launch path of the same decoder (``use_single_launch=
False``) over several steps, across ranks, state sizes, head dims, batch
sizes that give one or many work items per CTA, bf16, and graph capture;
plus: layers outside its range fall back, the workspace's barrier counters
are back at zero after every launch, and the bounded waits never fire.
The SISO step (one CTA per (batch row, head) state tile) is checked the same
way: against the oracle over several steps (state sizes, odd headdims,
rope_fraction 1.0, batches of one to many tiles per CTA), against the three
launches in fp32 and bf16, and under graph capture.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_params
from oracle import mamba3_oracle as orc
from src import _native as nat
from src.kernels.step import decode_step, prepare_decode_step
from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3

pytestmark = pytest.mark.gpu

SHAPES = [  # d_model, d_state, headdim, rank, batch
    (64, 16, 16, 1, 3),
    (64, 16, 16, 8, 5),
    (128, 32, 16, 2, 1),
    (256, 64, 32, 4, 128),
    (256, 64, 32, 4, 1000),
    (512, 128, 64, 8, 7),
    (512, 128, 128, 4, 33),
    (1024, 128, 64, 4, 64),
]


def _layer(d_model, d_state, headdim, R, seed, dtype=torch.float32):
    kw = dict(d_model=d_model, d_state=d_state, headdim=headdim, is_mimo=True, mimo_rank=R)
    dims = orc.layer_dims(**kw)
    params = orc.synthetic_params(dims, seed, bf16=dtype == torch.bfloat16, randomize_small=True)
    model = Mamba3(**kw, device="cuda", dtype=dtype)
    load_params(model, params)
    return kw, dims, params, model


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "d%d_n%d_p%d_r%d_b%d" % s)
def test_single_launch_matches_oracle(shape):
    d_model, D, P, R, B = shape
    kw, dims, params, model = _layer(d_model, D, P, R, seed=sum(shape))
    st = Mamba3Decoder(model, use_triton=False).init_state(B, device="cuda")
    launch = prepare_decode_step(model, st)  # the kernel itself, at any batch size
    assert launch is not None
    st_np = orc.init_state(dims, B)
    u = orc.synthetic_inputs(dims, B, 4, seed=7)
    with torch.no_grad():
        for t in range(4):
            o = launch.run(torch.from_numpy(u[t]).cuda())
            oe, st_np = orc.decode_step(u[t], params, dims, st_np)
            np.testing.assert_allclose(o.cpu().numpy(), oe, rtol=1e-4, atol=1e-4, err_msg=f"step {t}")
    for k in st_np:
        np.testing.assert_allclose(st[k].cpu().numpy(), st_np[k], rtol=1e-4, atol=1e-4, err_msg=k)
    assert nat.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES[1:7:2], ids=lambda s: "d%d_n%d_p%d_r%d_b%d" % s)
def test_single_launch_matches_three_launches(shape, dtype):
    d_model, D, P, R, B = shape
    _, _, _, model = _layer(d_model, D, P, R, seed=3, dtype=dtype)
    one = Mamba3Decoder(model, use_triton_full_fused=True)
    three = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    s1, s3 = one.init_state(B, device="cuda"), three.init_state(B, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    with torch.no_grad():
        for _ in range(6):
            u = torch.randn(B, d_model, device="cuda", generator=g).to(dtype)
            o1, s1 = one.step(u, s1)
            o3, s3 = three.step(u, s3)
            assert o1.dtype == o3.dtype == dtype
            torch.testing.assert_close(o1.float(), o3.float(), **tol)
    assert one._step_cache[1] is not None and three._step_cache is None
    for k in s1:
        torch.testing.assert_close(s1[k], s3[k], **tol)


def test_graph_capture_of_the_single_launch():
    """The single launch replays correctly from a CUDA graph that a caller
    captures around it; the decoder's own captured step takes the three
    launches, which replay faster."""
    _, dims, params, model = _layer(256, 64, 32, 4, seed=21)
    B = 128
    st = Mamba3Decoder(model, use_triton=False).init_state(B, device="cuda")
    launch = prepare_decode_step(model, st)
    u_static = torch.zeros(B, 256, device="cuda")
    st_np = orc.init_state(dims, B)
    with torch.no_grad():
        launch.run(u_static)  # one eager call before capture
        _, st_np = orc.decode_step(np.zeros((B, 256), np.float32), params, dims, st_np)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = launch.run(u_static)
        u = orc.synthetic_inputs(dims, B, 12, seed=22)
        for t in range(12):
            u_static.copy_(torch.from_numpy(u[t]))
            g.replay()
            oe, st_np = orc.decode_step(u[t], params, dims, st_np)
            np.testing.assert_allclose(out.cpu().numpy(), oe, rtol=1e-4, atol=1e-4, err_msg=f"step {t}")
    for k in st_np:
        np.testing.assert_allclose(st[k].cpu().numpy(), st_np[k], rtol=1e-4, atol=1e-4, err_msg=k)
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    dec.warmup_cuda_graph(dec.init_state(B, device="cuda"), n_warmup=1)
    assert dec._step_cache[1] is None
    assert nat.device_error() == 0


def test_barrier_words_advance_by_two_grids():
    """The grid barriers' words are never reset: after every launch the base
    word equals the arrival counter, and each launch adds the same amount."""
    _, dims, _, model = _layer(256, 64, 32, 4, seed=2)
    st = Mamba3Decoder(model, use_triton=False).init_state(300, device="cuda")
    launch = prepare_decode_step(model, st)
    u = torch.randn(300, 256, device="cuda")
    words = []
    for _ in range(3):
        launch.run(u)
        torch.cuda.synchronize()
        w = launch.workspace[:256].view(torch.int32).cpu()
        assert int(w[0]) == int(w[32]), "base word and arrival counter disagree"
        words.append(int(w[0]))
    step = words[1] - words[0]
    assert step > 0 and step % 2 == 0 and words[2] - words[1] == step
    assert nat.device_error() == 0


def test_decoder_reports_and_recovers_from_a_barrier_timeout():
    """A base word that the arrival counter can never reach makes the step's
    grid barriers wait out their bound (every CTA is resident, so nothing
    faults or hangs; the kernel records the timeout and returns).  The
    decoder's check raises, clears the error word and zeroes the workspace,
    after which the same decoder, workspace and state tensors (zeroed) decode
    correctly again."""
    _, dims, params, model = _layer(256, 64, 32, 4, seed=6)
    dec = Mamba3Decoder(model, use_triton_full_fused=True)
    st = dec.init_state(8, device="cuda")
    u = orc.synthetic_inputs(dims, 8, 3, 1)
    assert nat.device_error(reset=True) == 0
    with torch.no_grad():
        dec.step(torch.from_numpy(u[0]).cuda(), st)
        launch = dec._step_cache[1]
        assert launch is not None
        torch.cuda.synchronize()
        dec.check_device_error()  # nothing to report yet
        base = launch.workspace[:4].view(torch.int32)
        base.fill_(0x40000000)  # far ahead of the arrival counter
        dec.step(torch.from_numpy(u[1]).cuda(), st)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="bounded wait"):
            dec.check_device_error()
        assert nat.device_error() == 0
        assert int(launch.workspace.view(torch.int32)[:64].abs().sum()) == 0
        # recovered: the same workspace and state tensors (zeroed in place)
        # decode like the oracle again
        for v in st.values():
            v.zero_()
        st_np = orc.init_state(dims, 8)
        for t in range(3):
            o, st = dec.step(torch.from_numpy(u[t]).cuda(), st)
            oe, st_np = orc.decode_step(u[t], params, dims, st_np)
            np.testing.assert_allclose(o.cpu().numpy(), oe, rtol=1e-4, atol=1e-4, err_msg=f"step {t}")
        assert dec._step_cache[1] is launch
    assert nat.device_error() == 0


def test_decoder_policy_bounds_the_projection_work():
    from src.models.inference import SINGLE_LAUNCH_MAX_BATCH, single_launch_preferred
    _, _, _, small = _layer(64, 16, 16, 2, seed=4)
    for B, expect in ((SINGLE_LAUNCH_MAX_BATCH, True), (SINGLE_LAUNCH_MAX_BATCH + 1, False)):
        assert single_launch_preferred(small, B) == expect
        dec = Mamba3Decoder(small, use_triton_full_fused=True)
        st = dec.init_state(B, device="cuda")
        with torch.no_grad():
            dec.step(torch.randn(B, 64, device="cuda"), st)
        assert (dec._step_cache[1] is not None) == expect, B
    # a wide bf16 layer: large projections go to cuBLAS even at small batch
    _, _, _, wide = _layer(512, 128, 64, 8, seed=5, dtype=torch.bfloat16)
    assert single_launch_preferred(wide, 8) and not single_launch_preferred(wide, 128)


def test_layers_outside_the_range_fall_back():
    # 4 heads (not a multiple of 8): three-launch path, same results as eager
    model = Mamba3(d_model=32, d_state=16, headdim=16, is_mimo=True, mimo_rank=2, device="cuda")
    dec = Mamba3Decoder(model, use_triton_full_fused=True)
    ref = Mamba3Decoder(model, use_triton=False)
    s, sr = dec.init_state(2, device="cuda"), ref.init_state(2, device="cuda")
    u = torch.randn(2, 32, device="cuda")
    with torch.no_grad():
        o, s = dec.step(u, s)
        orf, sr = ref.step(u, sr)
    assert dec._step_cache[1] is None
    torch.testing.assert_close(o, orf, rtol=1e-4, atol=1e-4)
    with pytest.raises(ValueError):
        decode_step(model, u, s)
    # a SISO layer whose d_model is not a multiple of 4 is not taken
    siso = Mamba3(d_model=66, d_state=16, headdim=12, device="cuda")
    st = Mamba3Decoder(siso, use_triton=False).init_state(1, device="cuda")
    assert prepare_decode_step(siso, st) is None


# ---------------------------------------------------------------------------
# the SISO single launch (m3_siso_step)
# ---------------------------------------------------------------------------

SISO_SHAPES = [  # d_model, d_state, headdim, batch, rope_fraction
    (256, 64, 32, 1, 0.5),     # the reference's SISO d256 benchmark layer at batch 1
    (256, 64, 32, 8, 0.5),
    (64, 16, 16, 3, 0.5),
    (128, 32, 16, 2, 1.0),
    (96, 48, 24, 5, 0.5),      # headdim and d_state not powers of two
    (512, 128, 64, 4, 0.5),
    (256, 256, 64, 2, 0.5),
    (256, 64, 32, 64, 0.5),    # more tiles (1024) than CTAs
]


def _siso_layer(d_model, d_state, headdim, rope, seed, dtype=torch.float32):
    kw = dict(d_model=d_model, d_state=d_state, headdim=headdim, rope_fraction=rope)
    dims = orc.layer_dims(**kw)
    params = orc.synthetic_params(dims, seed, bf16=dtype == torch.bfloat16, randomize_small=True)
    model = Mamba3(**kw, device="cuda", dtype=dtype)
    load_params(model, params)
    return dims, params, model


@pytest.mark.parametrize("shape", SISO_SHAPES, ids=lambda s: "d%d_n%d_p%d_b%d_rope%s" % s)
def test_siso_single_launch_matches_oracle(shape):
    d_model, D, P, B, rope = shape
    dims, params, model = _siso_layer(d_model, D, P, rope, seed=40 + D + P + B)
    st = Mamba3Decoder(model, use_triton=False).init_state(B, device="cuda")
    launch = prepare_decode_step(model, st)
    assert launch is not None and launch.name == "m3_siso_step"
    st_np = orc.init_state(dims, B)
    u = orc.synthetic_inputs(dims, B, 4, seed=8)
    with torch.no_grad():
        for t in range(4):
            o = launch.run(torch.from_numpy(u[t]).cuda())
            oe, st_np = orc.decode_step(u[t], params, dims, st_np)
            np.testing.assert_allclose(o.cpu().numpy(), oe, rtol=1e-4, atol=1e-4, err_msg=f"step {t}")
    for k in st_np:
        np.testing.assert_allclose(st[k].cpu().numpy(), st_np[k], rtol=1e-4, atol=1e-4, err_msg=k)
    assert nat.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_siso_single_launch_matches_three_launches(dtype):
    """The single launch against the decoder's three launches (which the
    decoder keeps for SISO layers) on the same weights and inputs."""
    _, _, model = _siso_layer(256, 64, 32, 0.5, seed=9, dtype=dtype)
    three = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    B = 4
    s1, s3 = three.init_state(B, device="cuda"), three.init_state(B, device="cuda")
    one = prepare_decode_step(model, s1)
    g = torch.Generator(device="cuda").manual_seed(11)
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    with torch.no_grad():
        for _ in range(6):
            u = torch.randn(B, 256, device="cuda", generator=g).to(dtype)
            o1 = one.run(u)
            o3, s3 = three.step(u, s3)
            assert o1.dtype == o3.dtype == dtype
            torch.testing.assert_close(o1.float(), o3.float(), **tol)
    assert three._step_cache is None
    for k in s1:
        torch.testing.assert_close(s1[k], s3[k], **tol)


def test_siso_single_launch_in_a_graph():
    dims, params, model = _siso_layer(256, 64, 32, 0.5, seed=12)
    B = 2
    st = Mamba3Decoder(model, use_triton=False).init_state(B, device="cuda")
    launch = prepare_decode_step(model, st)
    u_static = torch.zeros(B, 256, device="cuda")
    out_static = torch.empty(B, 256, device="cuda")
    launch.run(u_static, out_static)  # the first call on the device happens before capture
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        launch.run(u_static, out_static)
    st_np = orc.init_state(dims, B)
    _, st_np = orc.decode_step(np.zeros((B, 256), np.float32), params, dims, st_np)
    u = orc.synthetic_inputs(dims, B, 8, seed=13)
    with torch.no_grad():
        for t in range(8):
            u_static.copy_(torch.from_numpy(u[t]))
            g.replay()
            oe, st_np = orc.decode_step(u[t], params, dims, st_np)
            np.testing.assert_allclose(out_static.cpu().numpy(), oe, rtol=1e-4, atol=1e-4, err_msg=f"step {t}")
    for k in st_np:
        np.testing.assert_allclose(st[k].cpu().numpy(), st_np[k], rtol=1e-4, atol=1e-4, err_msg=k)
    # the decoder: the single launch in eager steps, three launches in its graph
    from src.models.inference import single_launch_preferred
    assert single_launch_preferred(model, 1) and not single_launch_preferred(model, 1, graph=True)
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    st2 = dec.init_state(B, device="cuda")
    dec.warmup_cuda_graph(st2, n_warmup=1)
    assert dec._step_cache[1] is None
    eager = Mamba3Decoder(model, use_triton_full_fused=True)
    st3 = eager.init_state(B, device="cuda")
    with torch.no_grad():
        eager.step(torch.zeros(B, 256, device="cuda"), st3)
    assert eager._step_cache[1] is not None and eager._step_cache[1].name == "m3_siso_step"

