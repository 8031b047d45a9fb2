"""CPU oracle for the Mamba-3 single-token decode step (numpy, float32).

TEST INFRASTRUCTURE ONLY.  This module restates, in plain numpy, the
arithmetic of the reference PyTorch decode path of
michaelYZh/mamba3-fused-triton-kernel so that the CUDA path can be checked
against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``
(its ``cpu_baseline`` leg and ``--impl reference`` arm) may import it, and
only as the checker / the timed CPU restatement.  The shipped package never
imports it.

Every function cites the reference file:line it follows (paths relative to
the reference project root).  All arithmetic is float32, in the same
operation order as the reference PyTorch code.  bfloat16 models are emulated
by holding bf16-representable values in float32 arrays and rounding with
round-to-nearest-even exactly where the reference casts to bf16 (the
``in_proj`` output, the ``out_proj`` input and output).

Parity of this restatement is pinned by ``tests/test_oracle_golden.py``
against fixtures produced by running the reference itself
(``tests/golden/make_golden.py``) and against the reference tests' closed
forms and known answers.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
RMS_EPS = 1e-5          # src/models/mamba3.py:29 (RMSNorm eps default)
SOFTPLUS_THRESHOLD = 20.0  # torch.nn.functional.softplus default threshold


# ---------------------------------------------------------------------------
# bf16 emulation
# ---------------------------------------------------------------------------

def round_bf16(a) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned
    as float32.  Standard RNE on the upper 16 bits of the IEEE-754 pattern;
    NaN stays NaN."""
    a = np.ascontiguousarray(a, dtype=F32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(F32)
    return np.where(np.isnan(a), a, out).astype(F32, copy=False)


# ---------------------------------------------------------------------------
# Layer geometry
# ---------------------------------------------------------------------------

def layer_dims(d_model: int, d_state: int = 128, expand: int = 2,
               headdim: int = 64, ngroups: int = 1,
               rope_fraction: float = 0.5, is_mimo: bool = False,
               mimo_rank: int = 4, A_floor: float = 1e-4) -> dict:
    """Derived sizes of one Mamba-3 layer (src/models/mamba3.py:87-114)."""
    d_inner = int(expand * d_model)
    if d_inner % headdim != 0:
        raise ValueError("d_inner must be a multiple of headdim")
    nheads = d_inner // headdim
    if rope_fraction not in (0.5, 1.0):
        raise ValueError("rope_fraction must be 0.5 or 1.0")
    split = int(d_state * rope_fraction)
    if split % 2 != 0:
        split -= 1
    n_angles = split // 2
    if n_angles <= 0:
        raise ValueError("d_state too small for RoPE")
    R = mimo_rank if is_mimo else 1
    d_in_proj = 2 * d_inner + 2 * d_state * ngroups * R + 3 * nheads + n_angles
    return dict(d_model=d_model, d_state=d_state, d_inner=d_inner,
                nheads=nheads, headdim=headdim, ngroups=ngroups,
                mimo_rank=R, is_mimo=bool(is_mimo), split=split,
                num_rope_angles=n_angles, d_in_proj=d_in_proj,
                A_floor=float(A_floor))


# ---------------------------------------------------------------------------
# Elementwise helpers (float32)
# ---------------------------------------------------------------------------

def softplus(x):
    """torch.nn.functional.softplus(beta=1, threshold=20): x above the
    threshold passes through, else log1p(exp(x))."""
    x = np.asarray(x, dtype=F32)
    safe = np.minimum(x, F32(SOFTPLUS_THRESHOLD))
    with np.errstate(over="ignore"):
        sp = np.log1p(np.exp(safe)).astype(F32, copy=False)
    return np.where(x > F32(SOFTPLUS_THRESHOLD), x, sp).astype(F32, copy=False)


def sigmoid(x):
    x = np.asarray(x, dtype=F32)
    with np.errstate(over="ignore"):
        return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32, copy=False)


def silu(x):
    x = np.asarray(x, dtype=F32)
    return (x * sigmoid(x)).astype(F32, copy=False)


def rms_norm(x, weight, eps: float = RMS_EPS):
    """src/models/mamba3.py:34-36: x / sqrt(mean(x^2) + eps) * weight."""
    x = np.asarray(x, dtype=F32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    rms = np.sqrt(ms + F32(eps)).astype(F32, copy=False)
    return (x / rms * np.asarray(weight, dtype=F32)).astype(F32, copy=False)


def apply_rope(x, angles):
    """src/kernels/utils.py:31-44: rotate interleaved pairs (2i, 2i+1) of x
    by angles[..., i]."""
    x = np.asarray(x, dtype=F32)
    angles = np.asarray(angles, dtype=F32)
    c = np.cos(angles).astype(F32, copy=False)
    s = np.sin(angles).astype(F32, copy=False)
    x1 = x[..., 0::2]
    x2 = x[..., 1::2]
    out = np.empty(np.broadcast_shapes(x.shape, x.shape[:-1] + (2 * c.shape[-1],)), dtype=F32)
    out[..., 0::2] = x1 * c - x2 * s
    out[..., 1::2] = x1 * s + x2 * c
    return out


def trapezoidal_blend(bx_curr, bx_prev, trap):
    """src/kernels/utils.py:51-66: (1-trap)*Bx + trap*0.5*(Bx + Bx_prev)."""
    bx_curr = np.asarray(bx_curr, dtype=F32)
    bx_prev = np.asarray(bx_prev, dtype=F32)
    trap = np.asarray(trap, dtype=F32)
    return ((F32(1.0) - trap) * bx_curr
            + trap * F32(0.5) * (bx_curr + bx_prev)).astype(F32, copy=False)


# ---------------------------------------------------------------------------
# SSM-only decode (the kernel-level API)
# ---------------------------------------------------------------------------

def siso_decode(x, B_proj, C_proj, ADT, DT, trap, D_skip, h, bx_prev):
    """src/kernels/utils.py:73-102.

    x (B,H,P); B_proj, C_proj (B,H,D); ADT, DT, trap (B,H); D_skip (H,);
    h, bx_prev (B,H,P,D).  Returns (y (B,H,P), h_new, bx_new) where bx_new
    is the current, unblended x*B.
    """
    x = np.asarray(x, dtype=F32)
    decay = np.exp(np.asarray(ADT, F32))[..., None, None]
    dt_e = np.asarray(DT, F32)[..., None, None]
    tr_e = np.asarray(trap, F32)[..., None, None]
    bx_curr = (x[..., :, None] * np.asarray(B_proj, F32)[..., None, :]).astype(F32, copy=False)
    blended = trapezoidal_blend(bx_curr, bx_prev, tr_e)
    h_new = (decay * np.asarray(h, F32) + dt_e * blended).astype(F32, copy=False)
    y = np.einsum("bhd,bhpd->bhp", np.asarray(C_proj, F32), h_new).astype(F32, copy=False)
    y = (y + np.asarray(D_skip, F32)[None, :, None] * x).astype(F32, copy=False)
    return y, h_new, bx_curr


def mimo_decode(x, B_proj, C_proj, ADT, DT, trap, D_skip, mimo_x, mimo_o,
                h, bx_prev):
    """src/kernels/utils.py:109-148.

    x (B,H,P); B_proj, C_proj (B,R,H,D); ADT, DT, trap (B,H); D_skip (H,);
    mimo_x, mimo_o (H,R,P); h, bx_prev (B,H,D).
    """
    x = np.asarray(x, dtype=F32)
    x_r = np.einsum("bhp,hrp->bhr", x, np.asarray(mimo_x, F32)).astype(F32, copy=False)
    bx_curr = np.einsum("bhr,brhd->bhd", x_r, np.asarray(B_proj, F32)).astype(F32, copy=False)
    tr_e = np.asarray(trap, F32)[..., None]
    blended = trapezoidal_blend(bx_curr, bx_prev, tr_e)
    h_new = (np.exp(np.asarray(ADT, F32))[..., None] * np.asarray(h, F32)
             + np.asarray(DT, F32)[..., None] * blended).astype(F32, copy=False)
    y_r = np.einsum("brhd,bhd->brh", np.asarray(C_proj, F32), h_new).astype(F32, copy=False)
    skip = (np.asarray(D_skip, F32)[None, None, :] * x_r.transpose(0, 2, 1)).astype(F32, copy=False)
    y = np.einsum("brh,hrp->bhp", (y_r + skip).astype(F32, copy=False),
                  np.asarray(mimo_o, F32)).astype(F32, copy=False)
    return y, h_new, bx_curr


# ---------------------------------------------------------------------------
# Full layer step
# ---------------------------------------------------------------------------

def split_zx(zx, dims: dict):
    """src/models/mamba3.py:165-194 (inference branch): split the in_proj
    output into z, x (B,H,P), B_raw, C_raw (B,R,G,D), dd_dt, dd_A, trap_raw
    (B,H) and angle_raw (B,A)."""
    zx = np.asarray(zx, dtype=F32)
    Bsz = zx.shape[0]
    H, P, D = dims["nheads"], dims["headdim"], dims["d_state"]
    R, G, di = dims["mimo_rank"], dims["ngroups"], dims["d_inner"]
    dbc = D * G * R
    offs = np.cumsum([0, di, di, dbc, dbc, H, H, H, dims["num_rope_angles"]])
    parts = [zx[:, offs[i]:offs[i + 1]] for i in range(8)]
    z = parts[0].reshape(Bsz, H, P)
    x = parts[1].reshape(Bsz, H, P)
    B_raw = parts[2].reshape(Bsz, R, G, D)
    C_raw = parts[3].reshape(Bsz, R, G, D)
    return z, x, B_raw, C_raw, parts[4], parts[5], parts[6], parts[7]


def compute_params(zx, params: dict, dims: dict):
    """src/models/mamba3.py:160-217 (L=None branch).

    Returns z, x, B_exp, C_exp (B,R,H,D), ADT, DT, trap (B,H), angle_raw.
    """
    z, x, B_raw, C_raw, dd_dt, dd_A, trap_raw, angle_raw = split_zx(zx, dims)
    H = dims["nheads"]
    A_floor = F32(dims["A_floor"])
    # A = -(softplus(dd_A).clamp(max=-A_floor)); clamp(max=m) == min(., m)
    A = -np.minimum(softplus(dd_A), -A_floor)
    DT = softplus(dd_dt + np.asarray(params["dt_bias"], F32))
    ADT = (A * DT).astype(F32, copy=False)
    trap = sigmoid(trap_raw)
    B_n = rms_norm(B_raw, params["B_norm_weight"])      # (B,R,G,D)
    C_n = rms_norm(C_raw, params["C_norm_weight"])
    if dims["ngroups"] != 1:
        raise NotImplementedError("the reference decode path expands a single group")
    B_exp = np.broadcast_to(B_n, (B_n.shape[0], B_n.shape[1], H, B_n.shape[3]))
    C_exp = np.broadcast_to(C_n, (C_n.shape[0], C_n.shape[1], H, C_n.shape[3]))
    # rearrange(B_bias, "h r d -> r h d")
    B_exp = np.ascontiguousarray(B_exp + np.transpose(np.asarray(params["B_bias"], F32), (1, 0, 2)), F32)
    C_exp = np.ascontiguousarray(C_exp + np.transpose(np.asarray(params["C_bias"], F32), (1, 0, 2)), F32)
    return z, x, B_exp, C_exp, ADT, DT, trap, angle_raw


def ssm_from_zx(zx, params: dict, dims: dict, angle_state, ssm_state, bx_prev):
    """Everything between in_proj and out_proj: src/models/mamba3.py:321-349,
    i.e. what the reference full-fused kernel computes
    (src/kernels/fused_full_decode.py:37-225 SISO, :296-566 MIMO).

    Returns (y_gated (B,H,P), angle_state, ssm_state, bx_prev) as new arrays.
    """
    z, x, B_exp, C_exp, ADT, DT, trap, angle_raw = compute_params(zx, params, dims)
    split = dims["split"]
    R = dims["mimo_rank"]
    delta = (np.asarray(angle_raw, F32)[:, None, :] * DT[:, :, None]).astype(F32, copy=False)
    angle_state = (np.asarray(angle_state, F32) + delta).astype(F32, copy=False)
    ang = angle_state[:, None]  # (B, 1, H, A): broadcasts over the R ranks
    B_proj = np.concatenate([apply_rope(B_exp[..., :split], ang), B_exp[..., split:]], axis=-1)
    C_proj = np.concatenate([apply_rope(C_exp[..., :split], ang), C_exp[..., split:]], axis=-1)
    if dims["is_mimo"]:
        y, h_new, bx_new = mimo_decode(x, B_proj, C_proj, ADT, DT, trap,
                                       params["D"], params["mimo_x"], params["mimo_o"],
                                       ssm_state, bx_prev)
    else:
        y, h_new, bx_new = siso_decode(x, B_proj[:, 0], C_proj[:, 0], ADT, DT, trap,
                                       params["D"], ssm_state, bx_prev)
    y = (y * silu(z)).astype(F32, copy=False)
    return y, angle_state, h_new, bx_new


def decode_step(u, params: dict, dims: dict, state: dict, bf16: bool = False):
    """One decode step of one layer: src/models/mamba3.py:306-353 as driven by
    src/models/inference.py:271-282.

    ``u`` (B, d_model).  ``state`` holds angle_state, ssm_state, bx_prev.
    With ``bf16`` the weights/inputs are taken as bf16 values and the in_proj
    output, the out_proj input and output are rounded to bf16.
    Returns (out (B, d_model), new_state dict).
    """
    u = np.asarray(u, dtype=F32)
    W_in = np.asarray(params["in_proj_weight"], F32)
    W_out = np.asarray(params["out_proj_weight"], F32)
    zx = (u @ W_in.T).astype(F32, copy=False)
    if bf16:
        zx = round_bf16(zx)
    y, a, h, bx = ssm_from_zx(zx, params, dims, state["angle_state"],
                              state["ssm_state"], state["bx_prev"])
    y = y.reshape(y.shape[0], -1)
    if bf16:
        y = round_bf16(y)
    out = (y @ W_out.T).astype(F32, copy=False)
    if bf16:
        out = round_bf16(out)
    return out, {"angle_state": a, "ssm_state": h, "bx_prev": bx}


def init_state(dims: dict, batch: int) -> dict:
    """src/models/mamba3.py:355-381: zero fp32 state."""
    H, P, D, A = dims["nheads"], dims["headdim"], dims["d_state"], dims["num_rope_angles"]
    shape = (batch, H, D) if dims["is_mimo"] else (batch, H, P, D)
    return {"angle_state": np.zeros((batch, H, A), F32),
            "ssm_state": np.zeros(shape, F32),
            "bx_prev": np.zeros(shape, F32)}


def residual_block_step(x, norm_weight, params, dims, state, bf16=False):
    """One residual block of a stacked decoder: x + mixer(RMSNorm(x))
    (src/models/mamba3.py:412-421, with the mixer run as a decode step)."""
    x = np.asarray(x, F32)
    xn = rms_norm(x, norm_weight)
    if bf16:
        xn = round_bf16(xn)
    out, st = decode_step(xn, params, dims, state, bf16=bf16)
    res = (x + out).astype(F32, copy=False)
    if bf16:
        res = round_bf16(res)
    return res, st


# ---------------------------------------------------------------------------
# Seeded synthetic parameters (shared by fixtures and tests)
# ---------------------------------------------------------------------------

def synthetic_params(dims: dict, seed: int, bf16: bool = False,
                     w_std: float = 0.02, randomize_small: bool = True) -> dict:
    """Deterministic parameters from numpy's PCG64 stream.

    Shapes and names follow the reference Mamba3 module
    (src/models/mamba3.py:115-158).  ``dt_bias`` follows the reference's
    inverse-softplus of a log-uniform dt in [1e-3, 1e-1] (:118-124).  With
    ``randomize_small`` the biases, norm weights, D and the MIMO projections
    are drawn at random (so per-head and per-rank indexing is exercised)
    instead of the reference's constant init.
    """
    rng = np.random.default_rng(seed)
    H, P, D, R = dims["nheads"], dims["headdim"], dims["d_state"], dims["mimo_rank"]
    dm, di, dip = dims["d_model"], dims["d_inner"], dims["d_in_proj"]

    def f32(a):
        a = np.asarray(a, dtype=F32)
        return round_bf16(a) if bf16 else a

    dt = np.exp(rng.random(H) * (np.log(0.1) - np.log(1e-3)) + np.log(1e-3))
    dt = np.maximum(dt, 1e-4)
    dt_bias = dt + np.log(-np.expm1(-dt))
    p = {
        "in_proj_weight": f32(rng.standard_normal((dip, dm)) * w_std),
        "out_proj_weight": f32(rng.standard_normal((dm, di)) * w_std),
        "dt_bias": f32(dt_bias),
    }
    if randomize_small:
        p["B_bias"] = f32(1.0 + 0.5 * rng.standard_normal((H, R, D)))
        p["C_bias"] = f32(1.0 + 0.5 * rng.standard_normal((H, R, D)))
        p["B_norm_weight"] = f32(1.0 + 0.2 * rng.standard_normal(D))
        p["C_norm_weight"] = f32(1.0 + 0.2 * rng.standard_normal(D))
        p["D"] = f32(1.0 + 0.5 * rng.standard_normal(H))
        if dims["is_mimo"]:
            p["mimo_x"] = f32(rng.standard_normal((H, R, P)) / R)
            p["mimo_o"] = f32(rng.standard_normal((H, R, P)) / R)
            p["mimo_z"] = f32(np.ones((H, R, P)))
    else:
        p["B_bias"] = f32(np.ones((H, R, D)))
        p["C_bias"] = f32(np.ones((H, R, D)))
        p["B_norm_weight"] = f32(np.ones(D))
        p["C_norm_weight"] = f32(np.ones(D))
        p["D"] = f32(np.ones(H))
        if dims["is_mimo"]:
            p["mimo_x"] = f32(np.ones((H, R, P)) / R)
            p["mimo_o"] = f32(np.ones((H, R, P)) / R)
            p["mimo_z"] = f32(np.ones((H, R, P)))
    return p


def synthetic_inputs(dims: dict, batch: int, steps: int, seed: int,
                     bf16: bool = False) -> np.ndarray:
    """Token embeddings u_t ~ N(0, 1), shape (steps, batch, d_model)."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((steps, batch, dims["d_model"])).astype(F32, copy=False)
    return round_bf16(u) if bf16 else u


def ssm_kernel_inputs(kind: str, B: int, H: int, P: int, D: int, R: int,
                      seed: int, trap_value=None) -> dict:
    """Inputs shaped like the reference kernel tests
    (src/tests/test_siso.py:29-44, src/tests/test_mimo.py:29-47):
    negative A_log * dt decay, softmax dt + 0.01, sigmoid gate, random state.
    """
    rng = np.random.default_rng(seed)
    g = lambda *s: rng.standard_normal(s).astype(F32, copy=False)
    A_log = (-rng.random(H) * 2).astype(F32, copy=False)
    logits = g(B, H)
    e = np.exp(logits - logits.max(axis=-1, keepdims=True))
    dt = (e / e.sum(axis=-1, keepdims=True) + 0.01).astype(F32, copy=False)
    trap = sigmoid(g(B, H)) if trap_value is None else np.full((B, H), trap_value, F32)
    d = {"x": g(B, H, P), "ADT": (A_log[None, :] * dt).astype(F32, copy=False), "DT": dt,
         "trap": trap, "D_skip": g(H), "z": g(B, H, P)}
    if kind == "siso":
        d.update(B_proj=g(B, H, D), C_proj=g(B, H, D), h=g(B, H, P, D), bx_prev=g(B, H, P, D))
    else:
        d.update(B_proj=g(B, R, H, D), C_proj=g(B, R, H, D), h=g(B, H, D), bx_prev=g(B, H, D),
                 mimo_x=g(H, R, P), mimo_o=g(H, R, P))
    return d
