"""GPU test of ``Mamba3Decoder.step_host``: decode steps from and to pinned
host memory give the device path's results, on the single-launch kernel
(output stored straight into host memory; compared with eager steps, which
take the same kernel) and on the three-launch path (compared with captured
steps)."""

from __future__ import annotations

import pytest
import torch

from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("single", [True, False])
def test_step_host_matches_device_steps(single):
    torch.manual_seed(0)
    model = Mamba3(d_model=256, d_state=64, headdim=32, is_mimo=True, mimo_rank=4, device="cuda")
    a = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True, use_single_launch=single)
    b = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=not single, use_single_launch=single)
    sa, sb = a.init_state(16, device="cuda"), b.init_state(16, device="cuda")
    a.warmup_cuda_graph(sa, n_warmup=1)
    if single:
        with torch.no_grad():
            b.step(torch.zeros(16, 256, device="cuda"), sb)  # a's warm-up step
    else:
        b.warmup_cuda_graph(sb, n_warmup=1)
    g = torch.Generator().manual_seed(3)
    with torch.no_grad():
        for _ in range(5):
            u = torch.randn(16, 256, generator=g).pin_memory()
            oh = a.step_host(u)
            od, _ = b.step(u.cuda(), sb)
            assert oh.device.type == "cpu" and oh.is_pinned()
            torch.testing.assert_close(oh, od.cpu(), rtol=0, atol=0)
    assert (a._host_graph is not None) == single
    for k in sa:
        torch.testing.assert_close(sa[k], sb[k], rtol=0, atol=0)


def test_step_host_needs_a_graph_and_pinned_input():
    model = Mamba3(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2, device="cuda")
    dec = Mamba3Decoder(model, use_triton_full_fused=True)
    with pytest.raises(RuntimeError):
        dec.step_host(torch.zeros(1, 64).pin_memory())
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    dec.warmup_cuda_graph(dec.init_state(1, device="cuda"), n_warmup=1)
    with pytest.raises(AssertionError):
        dec.step_host(torch.zeros(1, 64))  # not pinned (checked at set-up)
    dec.step_host(torch.zeros(1, 64).pin_memory())
    with pytest.raises(AssertionError):
        dec.step_host(torch.zeros(2, 64).pin_memory())  # wrong shape


def test_step_host_of_a_large_layer_replays_the_captured_step():
    """Projection weights above STEP_HOST_SINGLE_MAX_WEIGHT_BYTES: step_host
    replays the captured three launches and copies the output back (faster
    there than the single launch's zero-copy rows), with the device path's
    results."""
    from src.models.inference import STEP_HOST_SINGLE_MAX_WEIGHT_BYTES
    torch.manual_seed(1)
    model = Mamba3(d_model=1024, d_state=128, headdim=64, is_mimo=True, mimo_rank=4, device="cuda")
    wbytes = (model.in_proj.weight.numel() + model.out_proj.weight.numel()) * 4
    assert wbytes > STEP_HOST_SINGLE_MAX_WEIGHT_BYTES
    a = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    b = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    sa, sb = a.init_state(2, device="cuda"), b.init_state(2, device="cuda")
    a.warmup_cuda_graph(sa, n_warmup=1)
    b.warmup_cuda_graph(sb, n_warmup=1)
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for _ in range(3):
            u = torch.randn(2, 1024, generator=g).pin_memory()
            oh = a.step_host(u)
            od, _ = b.step(u.cuda(), sb)
            torch.testing.assert_close(oh, od.cpu(), rtol=0, atol=0)
    assert a._host_graph is None
