"""SISO prefill (Mamba3Decoder.prefill on an is_mimo=False layer): one
in_proj GEMM over the whole prompt, ONE m3_siso_prefill launch (a CTA per
sequence and head, the head's state tile in registers from the first token
to the last) and one out_proj GEMM must give the outputs and the final
state of stepping the same prompt token by token -- and, in fp32, of the
oracle's decode loop -- across state widths (16 .. 256, one not a multiple
of 32), headdims, bf16, prompts of one token, prompts that are not a whole
number of the kernel's token chunks, many sequences and a non-zero
starting state; shapes outside the kernel's range step token by token."""

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

TAKEN = [  # d_model, d_state, headdim, batch, length, dtype
    (256, 64, 32, 3, 37, torch.float32),
    (512, 128, 64, 2, 9, torch.bfloat16),
    (256, 96, 32, 5, 1, torch.float32),
    (512, 128, 64, 40, 16, torch.float32),
    (512, 256, 64, 2, 7, torch.float32),
    (512, 256, 64, 1, 13, torch.bfloat16),
    (256, 16, 16, 2, 11, torch.float32),
    (2048, 128, 64, 2, 3, torch.bfloat16),
    (256, 64, 32, 1, 100, torch.float32),
]
DECLINED = [  # (3 * nheads + angles) * 4 bytes not a multiple of 16; a state tile over 64 floats a thread
    (128, 32, 128, 2, 4, torch.float32),
    (1024, 256, 128, 1, 3, torch.float32),
]


def _layer(d_model, D, P, dtype, seed):
    kw = dict(d_model=d_model, d_state=D, headdim=P, is_mimo=False)
    dims = orc.layer_dims(**kw)
    params = orc.synthetic_params(dims, seed, bf16=dtype == torch.bfloat16, randomize_small=True)
    model = Mamba3(**kw, device="cuda", dtype=dtype)
    load_params(model, params)
    return dims, params, model


def _run(case, expect_kernel):
    d_model, D, P, B, L, dtype = case
    dims, params, model = _layer(d_model, D, P, dtype, seed=sum(case[:5]))
    g = torch.Generator(device="cuda").manual_seed(11)
    u = torch.randn(B, L, d_model, device="cuda", generator=g).to(dtype)
    pre = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    ref = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    sp, sr = pre.init_state(B, device="cuda"), ref.init_state(B, device="cuda")
    with torch.no_grad():
        for t in range(2):  # start from a non-zero state
            w = torch.randn(B, d_model, device="cuda", generator=g).to(dtype)
            pre.step(w, sp)
            ref.step(w, sr)
        if expect_kernel:  # the prefill kernel, not the token-by-token fallback
            pre.step = lambda *a, **k: pytest.fail("prefill fell back to token steps")
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


@pytest.mark.parametrize("case", TAKEN, ids=lambda c: "d%d_n%d_p%d_b%d_l%d_%s" % (*c[:5], str(c[5])[6:]))
def test_siso_prefill_matches_token_steps(case):
    _run(case, expect_kernel=True)


@pytest.mark.parametrize("case", DECLINED, ids=lambda c: "d%d_n%d_p%d" % c[:3])
def test_siso_shapes_outside_the_kernel_step_token_by_token(case):
    _run(case, expect_kernel=False)


def test_siso_prefill_matches_the_oracle():
    dims, params, model = _layer(256, 64, 32, torch.float32, seed=79)
    B, L = 4, 12
    u = orc.synthetic_inputs(dims, B, L, seed=80)  # (L, B, d_model)
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


def test_siso_prefill_in_pieces_equals_one_prefill():
    # a prompt fed as 5 + 1 + 8 tokens ends in the state one prefill of 14 reaches
    dims, params, model = _layer(512, 128, 64, torch.float32, seed=81)
    B = 3
    u = torch.randn(B, 14, 512, device="cuda", generator=torch.Generator(device="cuda").manual_seed(12))
    dec = Mamba3Decoder(model, use_triton_full_fused=True)
    s1, s2 = dec.init_state(B, device="cuda"), dec.init_state(B, device="cuda")
    with torch.no_grad():
        o_all, s1 = dec.prefill(u, s1)
        parts = []
        for lo, hi in ((0, 5), (5, 6), (6, 14)):
            o, s2 = dec.prefill(u[:, lo:hi].contiguous(), s2)
            parts.append(o)
    torch.testing.assert_close(torch.cat(parts, dim=1), o_all, rtol=1e-5, atol=1e-5)
    for k in s1:
        torch.testing.assert_close(s1[k], s2[k], rtol=1e-5, atol=1e-5)
