"""Host-side model and API checks (CPU).

* ``Mamba3`` draws the same initial parameters as the reference for a seed
  (fixtures record the reference's own draws);
* the PyTorch reference path (``Mamba3Decoder(model, use_triton=False)``)
  reproduces the reference's decode outputs;
* CUDA backends refuse to run without a device instead of falling back.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import build_stack, golden_names, layer_kwargs, load_golden, load_params
from oracle import mamba3_oracle as orc
from src.kernels import utils as ku
from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3


@pytest.mark.parametrize("name", golden_names("init"))
def test_seeded_init_matches_reference(name):
    g = load_golden(name)
    torch.manual_seed(g["meta"]["seed"])
    model = Mamba3(**layer_kwargs(g["meta"]["layer"]))
    sd = model.state_dict()
    keys = sorted(k[4:] for k in g if k.startswith("sum."))
    assert sorted(sd) == keys
    for k in keys:
        v = sd[k].float().reshape(-1).numpy()
        np.testing.assert_array_equal(v[:8], g["head." + k])
        np.testing.assert_allclose(v.astype(np.float64).sum(), g["sum." + k], rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("name", [n for n in golden_names("layer") if not load_golden(n)["meta"]["bf16"]])
def test_pytorch_decoder_matches_reference(name):
    g = load_golden(name)
    m = g["meta"]
    model = Mamba3(**layer_kwargs(m["layer"]))
    dims = orc.layer_dims(**layer_kwargs(m["layer"]))
    load_params(model, orc.synthetic_params(dims, m["param_seed"]))
    dec = Mamba3Decoder(model, use_triton=False)
    u = orc.synthetic_inputs(dims, m["batch"], m["steps"], m["input_seed"])
    st = dec.init_state(m["batch"])
    with torch.no_grad():
        outs = [dec.step(torch.from_numpy(u[t]), st)[0].numpy() for t in range(m["steps"])]
    np.testing.assert_allclose(np.stack(outs), g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(st["angle_state"].numpy(), g["angle_state"], rtol=1e-6, atol=1e-6)
    if "ssm_state" in g:
        np.testing.assert_allclose(st["ssm_state"].numpy(), g["ssm_state"], rtol=1e-5, atol=1e-6)


def test_decode_sequence_and_forward_agree():
    torch.manual_seed(0)
    model = Mamba3(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2)
    u = torch.randn(2, 5, 64)
    with torch.no_grad():
        outs, _ = Mamba3Decoder(model, use_triton=False).decode_sequence(u)
        fwd = model(u)
    torch.testing.assert_close(outs, fwd)


def test_refs_match_oracle():
    d = orc.ssm_kernel_inputs("mimo", 2, 3, 8, 16, 4, 9)
    t = {k: torch.from_numpy(v) for k, v in d.items()}
    y, h, bx = ku.mamba3_mimo_decode_ref(t["x"], t["B_proj"], t["C_proj"], t["ADT"], t["DT"],
                                         t["trap"], t["D_skip"], t["mimo_x"], t["mimo_o"],
                                         t["h"], t["bx_prev"])
    y2, h2, bx2 = orc.mimo_decode(**{k: d[k] for k in ("x", "B_proj", "C_proj", "ADT", "DT", "trap",
                                                          "D_skip", "mimo_x", "mimo_o", "h", "bx_prev")})
    np.testing.assert_allclose(y.numpy(), y2, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(h.numpy(), h2, rtol=1e-6, atol=1e-6)
    x = torch.tensor([1.0, 0.0, 0.0, 1.0])
    ang = torch.tensor([0.0, torch.pi / 2])
    torch.testing.assert_close(ku.apply_rope(x, ang), torch.tensor([1.0, 0.0, -1.0, 0.0]),
                               atol=1e-6, rtol=0)
    assert ku._get_strides((2, 3, 4)) == [12, 4, 1]
    torch.testing.assert_close(ku.build_rope_freqs(4, "cpu"),
                               1.0 / (10000.0 ** (torch.arange(4.0) / 4)))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device behaviour")
@pytest.mark.parametrize("flags", [dict(), dict(use_triton_full_fused=True),
                                   dict(use_triton=False, use_triton_fused=True),
                                   dict(use_triton=False, use_compile=True)])
def test_cuda_backends_refuse_without_device(flags):
    model = Mamba3(d_model=64, d_state=16, headdim=16)
    with pytest.raises(RuntimeError, match="CUDA"):
        Mamba3Decoder(model, **flags)


def test_pytorch_backend_needs_no_device():
    model = Mamba3(d_model=64, d_state=16, headdim=16)
    dec = Mamba3Decoder(model, use_triton=False, use_cuda_graph=True)
    assert not dec.use_cuda_graph
    st = dec.init_state(3)
    assert st["ssm_state"].shape == (3, 8, 16, 16) and st["ssm_state"].dtype == torch.float32
    dec.warmup_cuda_graph(st)  # no-op without a CUDA backend
    out, st = dec.step(torch.randn(3, 64), st)
    assert out.shape == (3, 64)


@pytest.mark.parametrize("name", golden_names("stack"))
def test_stack_decoder_pytorch_matches_reference(name):
    """The stack decoder's PyTorch path reproduces the reference's own
    residual composition (tests/golden/stack3_*)."""
    from src.models.stack import Mamba3StackDecoder
    g = load_golden(name)
    m = g["meta"]
    dtype = torch.bfloat16 if m["bf16"] else torch.float32
    dims, blocks, _ = build_stack(m, dtype=dtype)
    dec = Mamba3StackDecoder(blocks, use_triton=False)
    st = dec.init_state(m["batch"])
    u = orc.synthetic_inputs(dims, m["batch"], m["steps"], m["seed"] + 100, bf16=m["bf16"])
    with torch.no_grad():
        outs = [dec.step(torch.from_numpy(u[t]).to(dtype), st)[0].float().numpy() for t in range(m["steps"])]
    np.testing.assert_allclose(np.stack(outs), g["out"], rtol=1e-2, atol=1e-2)


def test_prefill_on_the_pytorch_path_is_forward():
    """Mamba3Decoder.prefill from a zero state gives Mamba3.forward's outputs
    (the reference's sequential loop, src/models/mamba3.py:242-304)."""
    import torch as _t
    from src.models.inference import Mamba3Decoder as _Dec
    from src.models.mamba3 import Mamba3 as _M
    _t.manual_seed(3)
    m = _M(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2)
    u = _t.randn(2, 6, 64)
    dec = _Dec(m, use_triton=False)
    with _t.no_grad():
        out, st = dec.prefill(u, dec.init_state(2))
        ref = m(u)
    _t.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
