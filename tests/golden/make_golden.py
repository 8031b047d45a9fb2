"""Generate the golden decode fixtures by running the reference itself.

Run in a container that has the reference checkout (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py \
        --reference <reference checkout> --out tests/golden

For every case the weights and token embeddings come from the seeded numpy
generators in ``oracle/mamba3_oracle.py`` (``synthetic_params`` /
``synthetic_inputs`` / ``ssm_kernel_inputs``), so a test can rebuild the
same inputs without the reference and compare against the stored outputs.
The reference is driven through its public PyTorch decode path,
``Mamba3Decoder(model, use_triton=False).step`` (src/models/inference.py:271)
and its kernel references ``mamba3_siso_decode_ref`` /
``mamba3_mimo_decode_ref`` (src/kernels/utils.py:73,109), on the CPU.

Fixtures store per-step outputs, the per-step in_proj outputs (``zx``), the
final angle state and either the full final SSM state (small cases) or
per-(batch, head) sums and sums of squares of it (large cases).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import mamba3_oracle as orc  # noqa: E402

# name -> layer kwargs, batch, steps, bf16, param seed, input seed, full state?
LAYER_CASES = {
    "siso_tiny_f32": (dict(d_model=64, d_state=16, headdim=16), 3, 8, False, 100, 101, True),
    "siso_tiny_rope1_f32": (dict(d_model=64, d_state=16, headdim=16, rope_fraction=1.0,
                                 A_floor=1e-3), 2, 6, False, 110, 111, True),
    "mimo_tiny_r1_f32": (dict(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=1),
                         3, 8, False, 120, 121, True),
    "mimo_tiny_r2_f32": (dict(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2),
                         3, 8, False, 122, 123, True),
    "mimo_tiny_r4_f32": (dict(d_model=64, d_state=32, headdim=16, is_mimo=True, mimo_rank=4),
                         3, 8, False, 124, 125, True),
    "mimo_tiny_r8_f32": (dict(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=8),
                         3, 8, False, 126, 127, True),
    # the shapes of the reference's own SISO d256 / MIMO R4 d256 decode workloads
    "siso_d256_f32": (dict(d_model=256, d_state=64, headdim=32), 1, 16, False, 0, 1, False),
    "mimo_r4_d256_f32": (dict(d_model=256, d_state=64, headdim=32, is_mimo=True, mimo_rank=4),
                         4, 16, False, 0, 1, True),
    # the wide-layer shapes with bf16 projection weights
    "siso_d512_bf16": (dict(d_model=512, d_state=128, headdim=64), 2, 4, True, 2, 3, False),
    "mimo_r8_d512_bf16": (dict(d_model=512, d_state=128, headdim=64, is_mimo=True, mimo_rank=8),
                          2, 4, True, 4, 5, True),
}

# name -> kind, B, H, P, D, R, seed, trap value
SSM_CASES = {
    "ssm_siso_b2h4p16d64": ("siso", 2, 4, 16, 64, 1, 42, None),
    "ssm_siso_b2h4p32d128": ("siso", 2, 4, 32, 128, 1, 43, None),
    "ssm_siso_b2h4p64d64": ("siso", 2, 4, 64, 64, 1, 44, None),
    "ssm_siso_euler": ("siso", 1, 2, 8, 16, 1, 45, 0.0),
    "ssm_siso_trapezoid": ("siso", 1, 2, 8, 16, 1, 46, 1.0),
    "ssm_mimo_r1": ("mimo", 2, 4, 16, 64, 1, 50, None),
    "ssm_mimo_r2": ("mimo", 2, 4, 16, 64, 2, 51, None),
    "ssm_mimo_r4": ("mimo", 2, 4, 16, 64, 4, 52, None),
    "ssm_mimo_r8": ("mimo", 2, 4, 16, 64, 8, 53, None),
    "ssm_mimo_euler": ("mimo", 1, 2, 8, 16, 2, 54, 0.0),
    "ssm_mimo_trapezoid": ("mimo", 1, 2, 8, 16, 2, 55, 1.0),
}

# residual stack: layer kwargs, layers, batch, steps, bf16, seed
STACK_CASES = {
    "stack3_mimo_r4_bf16": (dict(d_model=64, d_state=32, headdim=16, is_mimo=True, mimo_rank=4),
                            3, 2, 4, True, 300),
}


def _ref_modules(reference: str):
    sys.path.insert(0, reference)
    import torch
    from src.models.mamba3 import Mamba3, RMSNorm
    from src.models.inference import Mamba3Decoder
    from src.kernels.utils import mamba3_siso_decode_ref, mamba3_mimo_decode_ref
    return torch, Mamba3, RMSNorm, Mamba3Decoder, mamba3_siso_decode_ref, mamba3_mimo_decode_ref


def _layer_kwargs(kw):
    keys = ("d_model", "d_state", "headdim", "rope_fraction", "is_mimo", "mimo_rank", "A_floor")
    return {k: kw[k] for k in keys if k in kw}


def _build_ref_model(torch, Mamba3, kw, params, bf16):
    dtype = torch.bfloat16 if bf16 else torch.float32
    model = Mamba3(**_layer_kwargs(kw), dtype=dtype)
    sd = {
        "in_proj.weight": params["in_proj_weight"], "out_proj.weight": params["out_proj_weight"],
        "dt_bias": params["dt_bias"], "B_bias": params["B_bias"], "C_bias": params["C_bias"],
        "B_norm.weight": params["B_norm_weight"], "C_norm.weight": params["C_norm_weight"],
        "D": params["D"],
    }
    for k in ("mimo_x", "mimo_z", "mimo_o"):
        if k in params:
            sd[k] = params[k]
    model.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)).to(dtype) for k, v in sd.items()})
    model.eval()
    return model


def _to_np(t):
    return t.detach().float().cpu().numpy().astype(np.float32)


def make_layer_case(mods, name, spec, out_dir):
    torch, Mamba3, _, Mamba3Decoder, _, _ = mods
    kw, batch, steps, bf16, pseed, iseed, full_state = spec
    dims = orc.layer_dims(**_layer_kwargs(kw))
    params = orc.synthetic_params(dims, pseed, bf16=bf16)
    u = orc.synthetic_inputs(dims, batch, steps, iseed, bf16=bf16)
    model = _build_ref_model(torch, Mamba3, kw, params, bf16)
    dec = Mamba3Decoder(model, use_triton=False)
    state = dec.init_state(batch)
    dtype = torch.bfloat16 if bf16 else torch.float32
    outs, zxs = [], []
    with torch.no_grad():
        for t in range(steps):
            ut = torch.from_numpy(u[t]).to(dtype)
            zxs.append(_to_np(model.in_proj(ut)))
            o, state = dec.step(ut, state)
            outs.append(_to_np(o))
    rec = {"out": np.stack(outs),
           "angle_state": _to_np(state["angle_state"]),
           "bx_sum": _to_np(state["bx_prev"]).reshape(batch, dims["nheads"], -1).sum(-1)}
    h = _to_np(state["ssm_state"])
    if full_state:
        rec["ssm_state"] = h
        rec["bx_prev"] = _to_np(state["bx_prev"])
    if bf16:
        # bf16 in_proj outputs: lets a test feed the reference's own zx to the fused path
        rec["zx"] = np.stack(zxs)
    rec["ssm_sum"] = h.reshape(batch, dims["nheads"], -1).sum(-1)
    rec["ssm_sumsq"] = (h.astype(np.float64) ** 2).reshape(batch, dims["nheads"], -1).sum(-1)
    meta = dict(kind="layer", layer=kw, batch=batch, steps=steps, bf16=bf16,
                param_seed=pseed, input_seed=iseed, full_state=full_state)
    np.savez_compressed(os.path.join(out_dir, name + ".npz"), meta=json.dumps(meta), **rec)


def make_ssm_case(mods, name, spec, out_dir):
    torch, _, _, _, siso_ref, mimo_ref = mods
    kind, B, H, P, D, R, seed, trap_value = spec
    d = orc.ssm_kernel_inputs(kind, B, H, P, D, R, seed, trap_value)
    T = {k: torch.from_numpy(v) for k, v in d.items()}
    if kind == "siso":
        y, h, bx = siso_ref(T["x"], T["B_proj"], T["C_proj"], T["ADT"], T["DT"], T["trap"],
                            T["D_skip"], T["h"], T["bx_prev"])
    else:
        y, h, bx = mimo_ref(T["x"], T["B_proj"], T["C_proj"], T["ADT"], T["DT"], T["trap"],
                            T["D_skip"], T["mimo_x"], T["mimo_o"], T["h"], T["bx_prev"])
    meta = dict(kind="ssm", ssm_kind=kind, B=B, H=H, P=P, D=D, R=R, seed=seed, trap_value=trap_value)
    h, bx = _to_np(h), _to_np(bx)
    rec = {"y": _to_np(y), "h_sum": h.sum(-1), "bx_sum": bx.sum(-1),
           "h_sumsq": (h.astype(np.float64) ** 2).sum(-1)}
    if h.size <= 32768:
        rec.update(h=h, bx=bx)
    np.savez_compressed(os.path.join(out_dir, name + ".npz"), meta=json.dumps(meta), **rec)


def make_stack_case(mods, name, spec, out_dir):
    torch, Mamba3, RMSNorm, Mamba3Decoder, _, _ = mods
    kw, layers, batch, steps, bf16, seed = spec
    dims = orc.layer_dims(**_layer_kwargs(kw))
    dtype = torch.bfloat16 if bf16 else torch.float32
    rng = np.random.default_rng(seed)
    decs, norms, states = [], [], []
    for l in range(layers):
        params = orc.synthetic_params(dims, seed + 1 + l, bf16=bf16)
        model = _build_ref_model(torch, Mamba3, kw, params, bf16)
        dec = Mamba3Decoder(model, use_triton=False)
        norm = RMSNorm(dims["d_model"])  # MambaBlock.norm: fp32 weight (src/models/mamba3.py:417)
        w = (1.0 + 0.2 * rng.standard_normal(dims["d_model"])).astype(np.float32)
        norm.weight.data.copy_(torch.from_numpy(w))
        decs.append(dec)
        norms.append(norm)
        states.append(dec.init_state(batch))
    u = orc.synthetic_inputs(dims, batch, steps, seed + 100, bf16=bf16)
    outs = []
    with torch.no_grad():
        for t in range(steps):
            x = torch.from_numpy(u[t]).to(dtype)
            for l in range(layers):
                o, states[l] = decs[l].step(norms[l](x), states[l])
                x = x + o
            outs.append(_to_np(x))
    meta = dict(kind="stack", layer=kw, layers=layers, batch=batch, steps=steps, bf16=bf16, seed=seed)
    np.savez_compressed(os.path.join(out_dir, name + ".npz"), meta=json.dumps(meta), out=np.stack(outs))


# language model (src/models/mamba3.py:396-481): config, batch, length, seed.
# The reference's own initialisation under torch.manual_seed(seed) (tied
# embeddings: the reference's lm_head only works tied) and its forward over a
# seeded token sequence; the fixture keeps the token ids, the logits and a
# sum per parameter (to check that a rebuilt model holds the same weights).
LM_CASES = {
    "lm2_mimo_r2": (dict(d_model=64, n_layer=2, vocab_size=50, d_intermediate=0,
                         ssm_cfg=dict(d_state=16, headdim=16, is_mimo=True, mimo_rank=2)), 2, 5, 410),
    "lm2_siso_mlp": (dict(d_model=64, n_layer=2, vocab_size=50, d_intermediate=32,
                          ssm_cfg=dict(d_state=16, headdim=16)), 2, 5, 411),
}


def make_lm_case(mods, name, spec, out_dir):
    torch = mods[0]
    from src.models.mamba3 import MambaConfig, MambaLMHeadModel
    cfg_kw, batch, length, seed = spec
    torch.manual_seed(seed)
    model = MambaLMHeadModel(MambaConfig(**cfg_kw)).eval()
    gen = torch.Generator().manual_seed(seed + 1)
    ids = torch.randint(0, cfg_kw["vocab_size"], (batch, length), generator=gen)
    with torch.no_grad():
        logits = model(ids)
    rec = {"input_ids": ids.numpy().astype(np.int64), "logits": _to_np(logits)}
    for pname, prm in model.state_dict().items():
        rec["sum." + pname] = np.array(_to_np(prm).reshape(-1).astype(np.float64).sum())
    meta = dict(kind="lm", config=cfg_kw, batch=batch, length=length, seed=seed)
    np.savez_compressed(os.path.join(out_dir, name + ".npz"), meta=json.dumps(meta), **rec)


# parameter initialisation under torch.manual_seed(seed) on the CPU
INIT_CASES = {
    "init_siso_d256": (dict(d_model=256, d_state=64, headdim=32), 0),
    "init_mimo_r4_d256": (dict(d_model=256, d_state=64, headdim=32, is_mimo=True, mimo_rank=4), 7),
}


def make_init_case(mods, name, spec, out_dir):
    torch, Mamba3 = mods[0], mods[1]
    kw, seed = spec
    torch.manual_seed(seed)
    model = Mamba3(**_layer_kwargs(kw))
    rec = {}
    for pname, prm in model.state_dict().items():
        v = _to_np(prm).reshape(-1)
        rec["sum." + pname] = np.array(v.astype(np.float64).sum())
        rec["head." + pname] = v[:8].copy()
    meta = dict(kind="init", layer=kw, seed=seed)
    np.savez_compressed(os.path.join(out_dir, name + ".npz"), meta=json.dumps(meta), **rec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (its src/ is imported)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    mods = _ref_modules(args.reference)
    torch = mods[0]
    torch.set_num_threads(1)
    for name, spec in LAYER_CASES.items():
        make_layer_case(mods, name, spec, args.out)
    for name, spec in SSM_CASES.items():
        make_ssm_case(mods, name, spec, args.out)
    for name, spec in STACK_CASES.items():
        make_stack_case(mods, name, spec, args.out)
    for name, spec in INIT_CASES.items():
        make_init_case(mods, name, spec, args.out)
    for name, spec in LM_CASES.items():
        make_lm_case(mods, name, spec, args.out)
    n = len(LAYER_CASES) + len(SSM_CASES) + len(STACK_CASES) + len(INIT_CASES) + len(LM_CASES)
    print("wrote", n, "fixtures to", args.out)


if __name__ == "__main__":
    main()
