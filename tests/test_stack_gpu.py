"""GPU checks of the stacked decode: the residual-add + RMSNorm kernel
against PyTorch, and the fused-backend stack decoder (whole stack in one
CUDA graph) against the reference fixture and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import build_stack, golden_names, load_golden
from oracle import mamba3_oracle as orc
from src.kernels.norm import residual_rmsnorm
from src.models.mamba3 import RMSNorm
from src.models.stack import Mamba3StackDecoder

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N", [(1, 64), (7, 2048), (256, 1000), (3, 8192), (5, 1001)])  # 1001: element-wise path
def test_residual_rmsnorm_matches_torch(dtype, M, N):
    g = torch.Generator(device="cuda").manual_seed(M + N)
    x = torch.randn(M, N, device="cuda", generator=g).to(dtype)
    o = torch.randn(M, N, device="cuda", generator=g).to(dtype)
    norm = RMSNorm(N).cuda()
    norm.weight.data.uniform_(0.5, 1.5)
    xo, xn = residual_rmsnorm(x, o, norm.weight)
    ref_x = x + o
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(xo, ref_x, rtol=0, atol=0)
    torch.testing.assert_close(xn.float(), norm(ref_x).float(), **tol)
    x2, xn2 = residual_rmsnorm(x, None, norm.weight)
    assert x2 is x
    torch.testing.assert_close(xn2.float(), norm(x).float(), **tol)
    xo3, none = residual_rmsnorm(x, o, None)
    assert none is None
    torch.testing.assert_close(xo3, ref_x, rtol=0, atol=0)


@pytest.mark.parametrize("name", golden_names("stack"))
def test_stack_decoder_graph_matches_reference(name):
    g = load_golden(name)
    m = g["meta"]
    dtype = torch.bfloat16 if m["bf16"] else torch.float32
    dims, blocks, _ = build_stack(m, device="cuda", dtype=dtype)
    dec = Mamba3StackDecoder(blocks, use_cuda_graph=True, use_triton_full_fused=True)
    st = dec.init_state(m["batch"], device="cuda")
    dec.warmup_cuda_graph(st, n_warmup=1)
    u = orc.synthetic_inputs(dims, m["batch"], m["steps"], m["seed"] + 100, bf16=m["bf16"])
    with torch.no_grad():
        outs = [dec.step(torch.from_numpy(u[t]).cuda().to(dtype), st)[0].float().cpu().numpy()
                for t in range(m["steps"])]
    np.testing.assert_allclose(np.stack(outs), g["out"], rtol=3e-2, atol=3e-2)


def test_fp32_stack_matches_oracle():
    """Four fp32 MIMO blocks, eight steps: the graph-captured fused stack vs
    the oracle's residual composition at 1e-4."""
    meta = dict(layer=dict(d_model=128, d_state=32, headdim=16, is_mimo=True, mimo_rank=4),
                layers=4, batch=3, steps=8, bf16=False, seed=900)
    dims, blocks, layers = build_stack(meta, device="cuda")
    dec = Mamba3StackDecoder(blocks, use_cuda_graph=True, use_triton_full_fused=True)
    st = dec.init_state(meta["batch"], device="cuda")
    dec.warmup_cuda_graph(st, n_warmup=2)
    ost = [orc.init_state(dims, meta["batch"]) for _ in layers]
    u = orc.synthetic_inputs(dims, meta["batch"], meta["steps"], 901)
    with torch.no_grad():
        for t in range(meta["steps"]):
            y, st = dec.step(torch.from_numpy(u[t]).cuda(), st)
            x = u[t]
            for l, (params, w) in enumerate(layers):
                x, ost[l] = orc.residual_block_step(x, w, params, dims, ost[l])
            np.testing.assert_allclose(y.cpu().numpy(), x, rtol=1e-4, atol=1e-4)
    for l in range(len(layers)):
        np.testing.assert_allclose(st[l]["ssm_state"].cpu().numpy(), ost[l]["ssm_state"], rtol=1e-4, atol=1e-4)
