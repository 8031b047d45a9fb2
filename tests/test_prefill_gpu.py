"""Prefill (Mamba3Decoder.prefill): a whole prompt through one in_proj GEMM,
ONE launch of the streamed kernel's prefill form (m3_mimo_prefill) and one
out_proj GEMM must give the outputs and the final state of stepping the
same prompt token by token -- and, in fp32, of the oracle's decode loop --
across ranks, state widths, headdims, bf16, prompts of one token, many
sequences, and a non-zero starting state; shapes outside the kernel's range
step token by token."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_params
from oracle import mamba3_oracle as orc
from src import _native as nat
from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3

pytestmark = pytest.mark.gpu

CASES = [  # d_model, d_state, headdim, R, batch, length, dtype
    (256, 64, 32, 4, 3, 37, torch.float32),
    (512, 128, 64, 8, 2, 9, torch.bfloat16),
    (256, 96, 32, 2, 5, 1, torch.float32),
    (512, 128, 64, 1, 40, 6, torch.float32),
    (1024, 256, 128, 4, 1, 5, torch.float32),
]


def _layer(d_model, D, P, R, dtype, seed):
    kw = dict(d_model=d_model, d_state=D, headdim=P, is_mimo=True, mimo_rank=R)
    dims = orc.layer_dims(**kw)
    params = orc.synthetic_params(dims, seed, bf16=dtype == torch.bfloat16, randomize_small=True)
    model = Mamba3(**kw, device="cuda", dtype=dtype)
    load_params(model, params)
    return dims, params, model


@pytest.mark.parametrize("case", CASES, ids=lambda c: "d%d_n%d_p%d_r%d_b%d_l%d_%s" % (*c[:6], str(c[6])[6:]))
def test_prefill_matches_token_steps(case):
    d_model, D, P, R, B, L, dtype = case
    dims, params, model = _layer(d_model, D, P, R, dtype, seed=sum(case[:6]))
    g = torch.Generator(device="cuda").manual_seed(9)
    u = torch.randn(B, L, d_model, device="cuda", generator=g).to(dtype)
    pre = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    ref = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    sp, sr = pre.init_state(B, device="cuda"), ref.init_state(B, device="cuda")
    with torch.no_grad():
        for t in range(2):  # start from a non-zero state
            w = torch.randn(B, d_model, device="cuda", generator=g).to(dtype)
            pre.step(w, sp)
            ref.step(w, sr)
        out, sp = pre.prefill(u, sp)
        outs = []
        for t in range(L):
            o, sr = ref.step(u[:, t].contiguous(), sr)
            outs.append(o.clone())
    ref_out = torch.stack(outs, dim=1)
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    assert out.shape == (B, L, d_model) and out.dtype == dtype
    torch.testing.assert_close(out.float(), ref_out.float(), **tol)
    for k in sp:
        torch.testing.assert_close(sp[k], sr[k], **tol)
    assert nat.device_error() == 0


def test_prefill_matches_the_oracle():
    dims, params, model = _layer(256, 64, 32, 4, torch.float32, seed=77)
    B, L = 4, 12
    u = orc.synthetic_inputs(dims, B, L, seed=78)  # (L, B, d_model)
    dec = Mamba3Decoder(model, use_triton_full_fused=True)
    st = dec.init_state(B, device="cuda")
    with torch.no_grad():
        out, st = dec.prefill(torch.from_numpy(np.ascontiguousarray(u.transpose(1, 0, 2))).cuda(), st)
    st_np = orc.init_state(dims, B)
    for t in range(L):
        oe, st_np = orc.decode_step(u[t], params, dims, st_np)
        np.testing.assert_allclose(out[:, t].cpu().numpy(), oe, rtol=1e-4, atol=1e-4, err_msg=f"token {t}")
    for k in st_np:
        np.testing.assert_allclose(st[k].cpu().numpy(), st_np[k], rtol=1e-4, atol=1e-4, err_msg=k)


def test_shapes_outside_the_kernel_step_token_by_token():
    # 4 heads (not a multiple of 8): the prefill kernel declines, the decoder steps
    model = Mamba3(d_model=32, d_state=16, headdim=16, is_mimo=True, mimo_rank=2, device="cuda")
    dec = Mamba3Decoder(model, use_triton_full_fused=True)
    ref = Mamba3Decoder(model, use_triton=False)
    u = torch.randn(2, 5, 32, device="cuda")
    s, sr = dec.init_state(2, device="cuda"), ref.init_state(2, device="cuda")
    with torch.no_grad():
        out, s = dec.prefill(u, s)
        out_r, sr = ref.prefill(u, sr)
    torch.testing.assert_close(out, out_r, rtol=1e-4, atol=1e-4)
