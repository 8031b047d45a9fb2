"""Decode-state I/O (src/state_io.py): the file format round-trips single
layers and stacks bit for bit, batch rows split and join back into the
original state, damaged files are refused with a clear error, and a decode
resumed from a saved file (PyTorch decode path, CPU) continues exactly like
the uninterrupted run."""

from __future__ import annotations

import os
import struct

import pytest
import torch

from src.models.inference import Mamba3Decoder
from src.models.mamba3 import Mamba3
from src.state_io import MAGIC, NAMES, concat_rows, load_states, save_states, slice_rows


def _state(B, H, P, D, A, mimo, seed):
    g = torch.Generator().manual_seed(seed)
    sh = (B, H, D) if mimo else (B, H, P, D)
    return {"angle_state": torch.randn(B, H, A, generator=g) * 100,
            "ssm_state": torch.randn(*sh, generator=g), "bx_prev": torch.randn(*sh, generator=g)}


def _equal(a, b):
    assert set(a) == set(b) == set(NAMES)
    for n in NAMES:
        assert a[n].dtype == b[n].dtype and torch.equal(a[n], b[n]), n


@pytest.mark.parametrize("mimo", [False, True])
def test_layer_round_trip(tmp_path, mimo):
    st = _state(5, 4, 8, 16, 4, mimo, seed=1)
    p = os.path.join(tmp_path, "s.m3state")
    save_states(p, st, meta={"step": 17})
    back, meta = load_states(p)
    _equal(back, st)
    assert meta == {"step": 17}
    with open(p, "rb") as f:
        assert f.read(8) == MAGIC


def test_stack_round_trip_and_rows(tmp_path):
    stack = [_state(7, 4, 8, 16, 4, True, seed=s) for s in range(3)]
    p = os.path.join(tmp_path, "stack.m3state")
    save_states(p, stack)
    back, _ = load_states(p)
    assert isinstance(back, list) and len(back) == 3
    for a, b in zip(back, stack):
        _equal(a, b)
    # a shard's rows leave and come back
    parts = [slice_rows(stack, 0, 3), slice_rows(stack, 3, 7)]
    for a, b in zip(concat_rows(parts), stack):
        _equal(a, b)
    one = slice_rows(stack[0], 2, 5)
    assert one["ssm_state"].shape[0] == 3 and one["ssm_state"].is_contiguous()


def test_damaged_files_are_refused(tmp_path):
    st = _state(2, 2, 4, 8, 2, True, seed=3)
    p = os.path.join(tmp_path, "s.m3state")
    save_states(p, st)
    raw = open(p, "rb").read()
    bad = os.path.join(tmp_path, "bad")
    open(bad, "wb").write(b"X" + raw[1:])
    with pytest.raises(ValueError, match="magic"):
        load_states(bad)
    open(bad, "wb").write(raw[:-8])
    with pytest.raises(ValueError, match="truncated"):
        load_states(bad)
    (hlen,) = struct.unpack("<Q", raw[8:16])
    open(bad, "wb").write(raw[:16] + raw[16:16 + hlen].replace(b'"version": 1', b'"version": 9') + raw[16 + hlen:])
    with pytest.raises(ValueError, match="version"):
        load_states(bad)
    with pytest.raises(ValueError, match="float32"):
        save_states(bad, {**st, "bx_prev": st["bx_prev"].double()})
    with pytest.raises(ValueError, match="batch"):
        save_states(bad, {**st, "ssm_state": st["ssm_state"][:1]})


def test_resume_through_a_file(tmp_path):
    """PyTorch decode path on CPU: 4 steps, save, load into a fresh decoder,
    4 more steps == 8 uninterrupted steps."""
    torch.manual_seed(0)
    model = Mamba3(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2)
    us = torch.randn(8, 3, 64)
    dec = Mamba3Decoder(model, use_triton=False)
    st = dec.init_state(3)
    with torch.no_grad():
        for t in range(4):
            dec.step(us[t], st)
        p = os.path.join(tmp_path, "resume.m3state")
        save_states(p, st, meta={"tokens": 4})
        for t in range(4, 8):
            o_full, st = dec.step(us[t], st)
        st2, meta = load_states(p)
        assert meta["tokens"] == 4
        dec2 = Mamba3Decoder(model, use_triton=False)
        for t in range(4, 8):
            o_res, st2 = dec2.step(us[t], st2)
    assert torch.equal(o_res, o_full)
    _equal(st2, st)
