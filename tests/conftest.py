"""Shared test set-up.

* registers the ``gpu`` marker (tests that need a B200 and the built CUDA
  library);
* puts the repository root (for ``oracle``) and the package directory (for
  the reference-compatible ``src`` package) on ``sys.path``;
* loads the golden fixtures written by ``tests/golden/make_golden.py``.
"""

from __future__ import annotations

import glob
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mamba3-fused-triton-kernel_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built sm_100a library")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        d = {k: z[k] for k in z.files}
    d["meta"] = json.loads(str(d["meta"]))
    return d


def golden_names(kind: str) -> list:
    out = []
    for f in sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))):
        name = os.path.basename(f)[:-4]
        if load_golden(name)["meta"]["kind"] == kind:
            out.append(name)
    return out


def layer_kwargs(kw: dict) -> dict:
    keys = ("d_model", "d_state", "headdim", "rope_fraction", "is_mimo", "mimo_rank", "A_floor")
    return {k: kw[k] for k in keys if k in kw}


def load_params(model, params: dict) -> None:
    """Load oracle-style numpy parameters into a ``Mamba3`` module."""
    import torch

    sd = {"in_proj.weight": params["in_proj_weight"], "out_proj.weight": params["out_proj_weight"],
          "dt_bias": params["dt_bias"], "B_bias": params["B_bias"], "C_bias": params["C_bias"],
          "B_norm.weight": params["B_norm_weight"], "C_norm.weight": params["C_norm_weight"],
          "D": params["D"]}
    for k in ("mimo_x", "mimo_z", "mimo_o"):
        if k in params:
            sd[k] = params[k]
    dtype = model.in_proj.weight.dtype
    dev = model.in_proj.weight.device
    model.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)).to(dev, dtype)
                           for k, v in sd.items()})


def build_stack(meta, device=None, dtype=None):
    """The residual-stack fixture's blocks (tests/golden/make_golden.py
    STACK_CASES): per layer synthetic parameters from seed + 1 + l and norm
    weights 1 + 0.2 N(0, 1) from the case seed."""
    import torch
    from oracle import mamba3_oracle as orc
    from src.models.mamba3 import MambaBlock
    dims = orc.layer_dims(**layer_kwargs(meta["layer"]))
    rng = np.random.default_rng(meta["seed"])
    blocks, oracle_layers = [], []
    kw = {k: v for k, v in layer_kwargs(meta["layer"]).items() if k != "d_model"}
    for l in range(meta["layers"]):
        params = orc.synthetic_params(dims, meta["seed"] + 1 + l, bf16=meta["bf16"])
        w = (1.0 + 0.2 * rng.standard_normal(dims["d_model"])).astype(np.float32)
        blk = MambaBlock(dims["d_model"], kw, device=device, dtype=dtype)
        load_params(blk.mixer, params)
        blk.norm.weight.data.copy_(torch.from_numpy(w))
        blocks.append(blk)
        oracle_layers.append((params, w))
    return dims, blocks, oracle_layers


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
