"""GPU tests of ``Mamba3Decoder`` with the CUDA backends.

Mirrors the reference's end-to-end check (src/tests/test_full_fused.py:
full-fused vs PyTorch eager, 1 step then 10 steps, tolerance 1e-3) and
asserts it for SISO and every MIMO rank, then adds: the reference fixtures,
CUDA-graph replay semantics (static output, in-place state), the partially
fused backends, a 1024-step drift bound (atol/rtol 1e-3 against the oracle),
bf16 weights, and resume from a saved state.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, layer_kwargs, load_golden, load_params
from oracle import mamba3_oracle as orc
from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3

pytestmark = pytest.mark.gpu


def _model(seed=0, dtype=torch.float32, **kw):
    torch.manual_seed(seed)
    return Mamba3(device="cuda", dtype=dtype, **kw)


def _max_diff(a, b):
    return (a.float() - b.float()).abs().max().item()


@pytest.mark.parametrize("mode,R", [("siso", 1), ("mimo", 1), ("mimo", 2), ("mimo", 4), ("mimo", 8)])
def test_full_fused_matches_pytorch_eager(mode, R):
    """src/tests/test_full_fused.py:10-102 as an asserting test."""
    model = _model(d_model=256, d_state=64, headdim=32, is_mimo=mode == "mimo", mimo_rank=R)
    ref = Mamba3Decoder(model, use_triton=False)
    fused = Mamba3Decoder(model, use_triton_full_fused=True)
    s_ref, s_fus = ref.init_state(2, device="cuda"), fused.init_state(2, device="cuda")
    torch.manual_seed(1)
    with torch.no_grad():
        u = torch.randn(2, 256, device="cuda")
        o_ref, s_ref = ref.step(u, s_ref)
        o_fus, s_fus = fused.step(u, s_fus)
        assert _max_diff(o_ref, o_fus) < 1e-3
        for _ in range(10):
            u = torch.randn(2, 256, device="cuda")
            o_ref, s_ref = ref.step(u, s_ref)
            o_fus, s_fus = fused.step(u, s_fus)
    assert _max_diff(o_ref, o_fus) < 1e-3
    for k in s_ref:
        torch.testing.assert_close(s_fus[k], s_ref[k], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("flags", [dict(use_triton=True), dict(use_triton_fused=True),
                                   dict(use_triton_full_fused=True)])
@pytest.mark.parametrize("mimo", [False, True])
def test_backends_against_reference_fixtures(flags, mimo):
    name = "mimo_r4_d256_f32" if mimo else "siso_d256_f32"
    g = load_golden(name)
    m = g["meta"]
    dims = orc.layer_dims(**layer_kwargs(m["layer"]))
    model = Mamba3(**layer_kwargs(m["layer"]), device="cuda")
    load_params(model, orc.synthetic_params(dims, m["param_seed"]))
    dec = Mamba3Decoder(model, **flags)
    u = orc.synthetic_inputs(dims, m["batch"], m["steps"], m["input_seed"])
    st = dec.init_state(m["batch"], device="cuda")
    with torch.no_grad():
        outs = [dec.step(torch.from_numpy(u[t]).cuda(), st)[0].cpu().numpy() for t in range(m["steps"])]
    np.testing.assert_allclose(np.stack(outs), g["out"], rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(st["angle_state"].cpu().numpy(), g["angle_state"], rtol=1e-4, atol=1e-5)
    if "ssm_state" in g:
        np.testing.assert_allclose(st["ssm_state"].cpu().numpy(), g["ssm_state"], rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("name", [n for n in golden_names("layer") if load_golden(n)["meta"]["bf16"]])
def test_bf16_decoder_against_reference_fixtures(name):
    g = load_golden(name)
    m = g["meta"]
    dims = orc.layer_dims(**layer_kwargs(m["layer"]))
    model = Mamba3(**layer_kwargs(m["layer"]), device="cuda", dtype=torch.bfloat16)
    load_params(model, orc.synthetic_params(dims, m["param_seed"], bf16=True))
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    st = dec.init_state(m["batch"], device="cuda")
    dec.warmup_cuda_graph(st, n_warmup=2)
    u = orc.synthetic_inputs(dims, m["batch"], m["steps"], m["input_seed"], bf16=True)
    outs = []
    with torch.no_grad():
        for t in range(m["steps"]):
            o, st = dec.step(torch.from_numpy(u[t]).cuda().bfloat16(), st)
            assert o.dtype == torch.bfloat16
            outs.append(o.float().cpu().numpy())
    # bf16 outputs: cuBLAS and the reference CPU GEMM may round the in_proj
    # output to neighbouring bf16 values; allow a few bf16 ulps.
    np.testing.assert_allclose(np.stack(outs), g["out"], rtol=3e-2, atol=3e-3)
    np.testing.assert_allclose(st["angle_state"].cpu().numpy(), g["angle_state"], rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("flags", [dict(use_triton_full_fused=True), dict(use_triton_fused=True),
                                   dict(use_triton=True)])
def test_cuda_graph_replay_semantics(flags):
    """src/models/inference.py:97-177: the graph replays in_proj -> kernel(s)
    -> out_proj, advances the captured state in place and returns the same
    static output buffer every step."""
    model = _model(d_model=256, d_state=64, headdim=32, is_mimo=True, mimo_rank=4)
    eager = Mamba3Decoder(model, **flags)
    graph = Mamba3Decoder(model, use_cuda_graph=True, **flags)
    s_e = eager.init_state(4, device="cuda")
    s_g = graph.init_state(4, device="cuda")
    ids = {k: id(v) for k, v in s_g.items()}
    ptrs = {k: v.data_ptr() for k, v in s_g.items()}
    graph.warmup_cuda_graph(s_g, n_warmup=3)
    for k in s_g:  # zero input from a zero state leaves the state at zero
        assert s_g[k].abs().max().item() == 0.0
    torch.manual_seed(2)
    outs = []
    with torch.no_grad():
        for _ in range(6):
            u = torch.randn(4, 256, device="cuda")
            o_e, s_e = eager.step(u, s_e)
            o_g, s_g2 = graph.step(u, s_g)
            outs.append(o_g)
            torch.testing.assert_close(o_g, o_e, rtol=1e-4, atol=1e-5)
    assert all(o.data_ptr() == outs[0].data_ptr() for o in outs)
    assert s_g2 is s_g and {k: id(v) for k, v in s_g.items()} == ids
    assert {k: v.data_ptr() for k, v in s_g.items()} == ptrs
    for k in s_e:
        torch.testing.assert_close(s_g[k], s_e[k], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("mimo", [False, True])
def test_partial_backends_match_pytorch(mimo):
    model = _model(d_model=128, d_state=32, headdim=32, is_mimo=mimo, mimo_rank=2)
    ref = Mamba3Decoder(model, use_triton=False)
    decs = [Mamba3Decoder(model, use_triton=True), Mamba3Decoder(model, use_triton_fused=True)]
    s_ref = ref.init_state(3, device="cuda")
    states = [d.init_state(3, device="cuda") for d in decs]
    torch.manual_seed(3)
    with torch.no_grad():
        for _ in range(8):
            u = torch.randn(3, 128, device="cuda")
            o_ref, s_ref = ref.step(u, s_ref)
            for d, s in zip(decs, states):
                o, _ = d.step(u, s)
                torch.testing.assert_close(o, o_ref, rtol=1e-4, atol=1e-5)
    for s in states:
        for k in s_ref:
            torch.testing.assert_close(s[k], s_ref[k], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("mode,R", [("siso", 1), ("mimo", 4), ("mimo", 8)])
def test_drift_1024_steps_against_oracle(mode, R):
    """1024 decode steps through the captured graph stay within atol/rtol 1e-3
    of the oracle (fp32), outputs and carried state."""
    kw = dict(d_model=256, d_state=64, headdim=32, is_mimo=mode == "mimo", mimo_rank=R)
    dims = orc.layer_dims(**kw)
    params = orc.synthetic_params(dims, 11, randomize_small=True)
    model = Mamba3(**kw, device="cuda")
    load_params(model, params)
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    B = 2
    st = dec.init_state(B, device="cuda")
    dec.warmup_cuda_graph(st, n_warmup=1)
    u = orc.synthetic_inputs(dims, B, 1024, 12)
    st_np = orc.init_state(dims, B)
    worst = 0.0
    with torch.no_grad():
        for t in range(1024):
            o, st = dec.step(torch.from_numpy(u[t]).cuda(), st)
            oe, st_np = orc.decode_step(u[t], params, dims, st_np)
            if t % 64 == 63 or t == 0:
                oc = o.cpu().numpy()
                np.testing.assert_allclose(oc, oe, rtol=1e-3, atol=1e-3, err_msg=f"step {t}")
                worst = max(worst, float(np.abs(oc - oe).max()))
    for k in st_np:
        np.testing.assert_allclose(st[k].cpu().numpy(), st_np[k], rtol=1e-3, atol=1e-3, err_msg=k)


@pytest.mark.parametrize("mimo", [False, True])
def test_bf16_weights_match_pytorch_bf16(mimo):
    """bf16 weights, 16 graph-replayed steps.  The fused path (for MIMO the
    single-launch kernel with its own projections) and PyTorch bf16 eager
    round differently, so both are measured against fp32 arithmetic on the
    same bf16 weights and inputs: the fused path's error must stay within
    twice PyTorch bf16's own, and the two within bf16 distance of each other."""
    import copy
    model = _model(d_model=512, d_state=128, headdim=64, is_mimo=mimo, mimo_rank=8, dtype=torch.bfloat16)
    ref = Mamba3Decoder(model, use_triton=False)
    ref32 = Mamba3Decoder(copy.deepcopy(model).float(), use_triton=False)
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    s_ref, s = ref.init_state(8, device="cuda"), dec.init_state(8, device="cuda")
    s32 = ref32.init_state(8, device="cuda")
    dec.warmup_cuda_graph(s, n_warmup=2)
    torch.manual_seed(4)
    with torch.no_grad():
        for _ in range(16):
            u = torch.randn(8, 512, device="cuda").bfloat16()
            o_ref, s_ref = ref.step(u, s_ref)
            o32, s32 = ref32.step(u.float(), s32)
            o, s = dec.step(u, s)
    assert o.dtype == torch.bfloat16
    err_ours, err_torch = _max_diff(o, o32), _max_diff(o_ref, o32)
    assert err_ours <= 2 * err_torch + 1e-3, (err_ours, err_torch)
    torch.testing.assert_close(o.float(), o_ref.float(), rtol=3e-2, atol=2e-2)
    torch.testing.assert_close(s["angle_state"], s_ref["angle_state"], rtol=1e-3, atol=1e-4)
    for k in ("ssm_state", "bx_prev"):
        e_ours, e_torch = _max_diff(s[k], s32[k]), _max_diff(s_ref[k], s32[k])
        assert e_ours <= 2 * e_torch + 1e-3, (k, e_ours, e_torch)
    torch.testing.assert_close(s["ssm_state"], s_ref["ssm_state"], rtol=2e-2, atol=1e-2)


def test_resume_from_saved_state():
    """Checkpoint/resume: a copy of the state after k steps, fed to a fresh
    decoder, continues exactly like the uninterrupted run (both on the
    three-launch path, which eager and captured steps then share)."""
    model = _model(d_model=256, d_state=64, headdim=32, is_mimo=True, mimo_rank=4)
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    torch.manual_seed(5)
    us = torch.randn(12, 3, 256, device="cuda")
    st = dec.init_state(3, device="cuda")
    with torch.no_grad():
        for t in range(6):
            dec.step(us[t], st)
        saved = {k: v.detach().cpu().clone() for k, v in st.items()}
        for t in range(6, 12):
            o_full, st = dec.step(us[t], st)
        dec2 = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True, use_single_launch=False)
        st2 = {k: v.cuda() for k, v in saved.items()}
        # warm-up steps would advance a non-zero state: capture with n_warmup=0
        dec2.warmup_cuda_graph(st2, n_warmup=0)
        for t in range(6, 12):
            o_res, st2 = dec2.step(us[t], st2)
    torch.testing.assert_close(o_res, o_full, rtol=1e-6, atol=1e-6)
    for k in st:
        torch.testing.assert_close(st2[k], st[k], rtol=1e-6, atol=1e-6)


def test_decode_sequence_graph_mode_keeps_every_output():
    model = _model(d_model=64, d_state=16, headdim=16)
    eager = Mamba3Decoder(model, use_triton_full_fused=True)
    graph = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    st = graph.init_state(2, device="cuda")
    graph.warmup_cuda_graph(st, n_warmup=1)
    u = torch.randn(2, 5, 64, device="cuda")
    with torch.no_grad():
        o_e, _ = eager.decode_sequence(u)
        o_g, _ = graph.decode_sequence(u, st)
    torch.testing.assert_close(o_g, o_e, rtol=1e-5, atol=1e-6)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_second_device_in_the_same_process():
    """Kernels launched with a dynamic shared memory opt-in (the streamed
    MIMO kernel, the SISO kernel, both prefill kernels) on cuda:1 after
    cuda:0 in one process: the opt-in is made per device, so each device's
    results match PyTorch eager on that device."""
    for dev in ("cuda:0", "cuda:1"):
        for mimo in (False, True):
            with torch.cuda.device(dev):
                torch.manual_seed(5)
                model = Mamba3(d_model=512, d_state=128, headdim=64, is_mimo=mimo, mimo_rank=4, device=dev)
                ref = Mamba3Decoder(model, use_triton=False)
                fused = Mamba3Decoder(model, use_triton_full_fused=True)
                B = 300
                s_ref, s = ref.init_state(B, device=dev), fused.init_state(B, device=dev)
                g = torch.Generator(device=dev).manual_seed(6)
                u = torch.randn(B, 4, 512, device=dev, generator=g)
                with torch.no_grad():
                    for t in range(4):
                        o_ref, s_ref = ref.step(u[:, t], s_ref)
                    o, s = fused.prefill(u, s)
                torch.testing.assert_close(o[:, -1], o_ref, rtol=1e-4, atol=1e-4)
                for k in s_ref:
                    torch.testing.assert_close(s[k], s_ref[k], rtol=1e-4, atol=1e-4)
                with torch.no_grad():
                    o_ref, s_ref = ref.step(u[:, 0], s_ref)
                    o, s = fused.step(u[:, 0], s)
                torch.testing.assert_close(o, o_ref, rtol=1e-4, atol=1e-4)
                assert o.device == torch.device(dev)
