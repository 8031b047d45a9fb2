"""Decode-state I/O on the CUDA decode path: a state saved to a file and
loaded back onto the GPU resumes a (graph-captured) decode exactly, and
batch rows decoded on two shards and then joined continue like a run that
held the whole batch from the start."""

from __future__ import annotations

import os

import pytest
import torch

from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3
from src.state_io import NAMES, concat_rows, load_states, save_states, slice_rows

pytestmark = pytest.mark.gpu


def _model():
    torch.manual_seed(11)
    return Mamba3(d_model=256, d_state=64, headdim=32, is_mimo=True, mimo_rank=4, device="cuda")


def test_resume_from_file_on_the_gpu(tmp_path):
    model = _model()
    us = torch.randn(10, 4, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))
    # eager and captured steps on the same (three-launch) path
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_single_launch=False)
    st = dec.init_state(4, device="cuda")
    p = os.path.join(tmp_path, "gpu.m3state")
    with torch.no_grad():
        for t in range(5):
            dec.step(us[t], st)
        save_states(p, st)
        for t in range(5, 10):
            o_full, st = dec.step(us[t], st)
        st2, _ = load_states(p, device="cuda")
        dec2 = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True, use_single_launch=False)
        dec2.warmup_cuda_graph(st2, n_warmup=0)
        for t in range(5, 10):
            o_res, st2 = dec2.step(us[t], st2)
    torch.testing.assert_close(o_res, o_full, rtol=1e-6, atol=1e-6)
    for n in NAMES:
        torch.testing.assert_close(st2[n], st[n], rtol=1e-6, atol=1e-6)


def test_shards_join_into_one_batch():
    model = _model()
    us = torch.randn(8, 6, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    full = Mamba3Decoder(model, use_triton_full_fused=True)
    sf = full.init_state(6, device="cuda")
    halves = [Mamba3Decoder(model, use_triton_full_fused=True) for _ in range(2)]
    sh = [h.init_state(3, device="cuda") for h in halves]
    with torch.no_grad():
        for t in range(4):
            full.step(us[t], sf)
            for r in range(2):
                halves[r].step(us[t, 3 * r:3 * r + 3], sh[r])
        joined = concat_rows([slice_rows(s, 0, 3) for s in sh])
        for t in range(4, 8):
            o_full, sf = full.step(us[t], sf)
            o_join, joined = full.step(us[t], joined)
    torch.testing.assert_close(o_join, o_full, rtol=1e-5, atol=1e-5)
    for n in NAMES:
        torch.testing.assert_close(joined[n], sf[n], rtol=1e-5, atol=1e-5)
