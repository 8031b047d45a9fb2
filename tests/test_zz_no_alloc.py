"""GPU test of m3_mimo_step_static, the decode step for callers that cannot
allocate device memory (a plugin given device buffers without access to its
host framework's allocator, a serving thread that must not call cudaMalloc,
a process whose device footprint is fixed after start-up).

The entry point runs the single-launch step on a scratch array inside the
library instead of a caller workspace.  Called through the C ABI, it must
give the results of m3_mimo_step (caller workspace) on the same inputs, on
two calls in a row (the second call finds the first call's leftovers in the
shared array), outputs and carried state alike.

This file is collected last so that a run stopping at its first failure has
run every other test already; it also passes alone in a fresh process.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_params
from oracle import mamba3_oracle as orc
from src import _native as nat
from src.kernels.step import prepare_decode_step
from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3

pytestmark = pytest.mark.gpu


def _layer(d_model, d_state, headdim, R, dtype, seed):
    kw = dict(d_model=d_model, d_state=d_state, headdim=headdim, is_mimo=True, mimo_rank=R)
    dims = orc.layer_dims(**kw)
    params = orc.synthetic_params(dims, seed, bf16=dtype == torch.bfloat16, randomize_small=True)
    model = Mamba3(**kw, device="cuda", dtype=dtype)
    load_params(model, params)
    return model


@pytest.mark.parametrize("dtype,shape", [(torch.float32, (256, 64, 32, 4, 128)),
                                         (torch.bfloat16, (512, 128, 64, 8, 7))],
                         ids=["f32_d256_r4_b128", "bf16_d512_r8_b7"])
def test_static_scratch_step_matches_workspace_step(dtype, shape):
    d_model, D, P, R, B = shape
    model = _layer(d_model, D, P, R, dtype, seed=41)
    ref = Mamba3Decoder(model, use_triton=False)
    s_ws, s_static = ref.init_state(B, device="cuda"), ref.init_state(B, device="cuda")
    launch = prepare_decode_step(model, s_ws)  # m3_mimo_step with its own workspace
    assert launch is not None
    lib = nat.load()
    stream = nat.stream_handle(torch.device("cuda"))
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    out_ws = torch.empty(B, d_model, device="cuda", dtype=dtype)
    out_static = torch.empty(B, d_model, device="cuda", dtype=dtype)
    g = torch.Generator(device="cuda").manual_seed(42)
    for call in range(2):
        u = torch.randn(B, d_model, device="cuda", generator=g).to(dtype)
        launch.run(u, out_ws)
        a = nat.StepArgs.from_buffer_copy(launch.args)  # same layer, inputs and strides ...
        a.ssm_state = s_static["ssm_state"].data_ptr()   # ... its own state and output,
        a.bx_prev = s_static["bx_prev"].data_ptr()
        a.angle_state = s_static["angle_state"].data_ptr()
        a.out, a.out_stride_b = out_static.data_ptr(), out_static.stride(0)
        a.workspace, a.workspace_bytes = None, 0            # and no workspace
        st = lib.m3_mimo_step_static(launch.dims, a, stream)
        assert st == nat.M3_OK, nat.status_string(st)
        torch.cuda.synchronize()
        torch.testing.assert_close(out_static.float(), out_ws.float(), **tol, msg=f"call {call}")
        for k in s_ws:
            torch.testing.assert_close(s_static[k], s_ws[k], **tol, msg=f"{k} after call {call}")
    assert nat.device_error() == 0


def test_static_scratch_rejects_a_batch_beyond_its_size():
    model = _layer(256, 64, 32, 4, torch.float32, seed=43)
    B = 4096
    st = Mamba3Decoder(model, use_triton=False).init_state(B, device="cuda")
    launch = prepare_decode_step(model, st)
    a = nat.StepArgs.from_buffer_copy(launch.args)
    u = torch.zeros(B, 256, device="cuda")
    out = torch.full((B, 256), 7.0, device="cuda")
    a.u, a.u_stride_b = u.data_ptr(), u.stride(0)
    a.out, a.out_stride_b = out.data_ptr(), out.stride(0)
    a.workspace, a.workspace_bytes = None, 0
    assert launch.workspace.numel() > nat.STEP_STATIC_SCRATCH_BYTES
    assert nat.load().m3_mimo_step_static(launch.dims, a, nat.stream_handle(u.device)) == nat.M3_ERR_SCRATCH
    torch.cuda.synchronize()
    assert bool((out == 7.0).all()), "a rejected call must not launch"
