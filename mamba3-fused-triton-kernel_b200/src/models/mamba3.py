"""Mamba-3 layer: parameters, PyTorch reference decode, state allocation.

Same constructor, attribute names, parameter names/shapes and parameter
initialisation order as the reference's ``src/models/mamba3.py`` (so a
``state_dict`` saved by one loads into the other, and the same
``torch.manual_seed`` gives the same weights).  ``Mamba3.step`` is the
PyTorch reference decode (``Mamba3Decoder(model, use_triton=False)``); the
CUDA backends live in ``src.models.inference`` and ``src.kernels``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from src.kernels.utils import apply_rope, mamba3_mimo_decode_ref, mamba3_siso_decode_ref


class RMSNorm(nn.Module):
    """x / sqrt(mean(x^2) + eps) * weight, computed in fp32 and returned in
    the input dtype (reference: src/models/mamba3.py:26-36)."""

    def __init__(self, d: int, eps: float = 1e-5, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d, device=device, dtype=dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        rms = xf.pow(2).mean(dim=-1, keepdim=True).add(self.eps).sqrt()
        return (xf / rms * self.weight.to(x.device)).to(x.dtype)


class Mamba3(nn.Module):
    """Mamba-3 sequence-mixing layer (reference: src/models/mamba3.py:39-389).

    ``d_inner = expand * d_model`` is split into ``nheads = d_inner / headdim``
    heads; each head carries a (headdim, d_state) state (SISO) or a
    (d_state,) state with ``mimo_rank`` input/output projections (MIMO).
    The first ``d_state * rope_fraction`` state entries (rounded down to even)
    are rotated by per-head accumulated angles (RoPE on B and C).
    """

    def __init__(self, d_model: int, d_state: int = 128, expand: int = 2, headdim: int = 64,
                 ngroups: int = 1, rope_fraction: float = 0.5, dt_min: float = 0.001,
                 dt_max: float = 0.1, dt_init_floor: float = 1e-4, A_floor: float = 1e-4,
                 is_mimo: bool = False, mimo_rank: int = 4, device=None, dtype=None):
        fk = {"device": device, "dtype": dtype}
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.expand = expand
        self.headdim = headdim
        self.A_floor = A_floor
        self.is_mimo = is_mimo
        self.mimo_rank = mimo_rank if is_mimo else 1
        self.num_bc_heads = ngroups

        self.d_inner = int(expand * d_model)
        assert self.d_inner % headdim == 0
        self.nheads = self.d_inner // headdim

        assert rope_fraction in (0.5, 1.0)
        split = int(d_state * rope_fraction)
        self.split_tensor_size = split - (split % 2)
        self.num_rope_angles = self.split_tensor_size // 2
        assert self.num_rope_angles > 0

        d_bc = d_state * ngroups * self.mimo_rank
        d_in_proj = 2 * self.d_inner + 2 * d_bc + 3 * self.nheads + self.num_rope_angles
        # Parameter creation order matches the reference so that a seeded
        # generator yields identical weights: in_proj, dt_bias, biases,
        # norms, MIMO projections, D, out_proj.
        self.in_proj = nn.Linear(d_model, d_in_proj, bias=False, **fk)

        log_lo, log_hi = math.log(dt_min), math.log(dt_max)
        dt = torch.exp(torch.rand(self.nheads, **fk) * (log_hi - log_lo) + log_lo)
        dt = dt.clamp(min=dt_init_floor)
        # inverse softplus: softplus(dt_bias) == dt
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        self.dt_bias._no_weight_decay = True

        self.B_bias = nn.Parameter(torch.ones(self.nheads, self.mimo_rank, d_state, **fk))
        self.C_bias = nn.Parameter(torch.ones(self.nheads, self.mimo_rank, d_state, **fk))
        self.B_bias._no_weight_decay = True
        self.C_bias._no_weight_decay = True

        self.B_norm = RMSNorm(d_state, **fk)
        self.C_norm = RMSNorm(d_state, **fk)

        if self.is_mimo:
            shape = (self.nheads, self.mimo_rank, headdim)
            self.mimo_x = nn.Parameter(torch.ones(*shape, **fk) / self.mimo_rank)
            self.mimo_z = nn.Parameter(torch.ones(*shape, **fk))
            self.mimo_o = nn.Parameter(torch.ones(*shape, **fk) / self.mimo_rank)

        self.D = nn.Parameter(torch.ones(self.nheads, **fk))
        self.D._no_weight_decay = True

        self.out_proj = nn.Linear(self.d_inner, d_model, bias=False, **fk)

    # ------------------------------------------------------------------
    # geometry of the in_proj output
    # ------------------------------------------------------------------

    @property
    def d_in_proj(self) -> int:
        return self.in_proj.out_features

    def split_sizes(self) -> list:
        """Column sizes of [z | x | B | C | dd_dt | dd_A | trap | angle]
        (reference: src/models/mamba3.py:165-179)."""
        d_bc = self.d_state * self.num_bc_heads * self.mimo_rank
        H = self.nheads
        return [self.d_inner, self.d_inner, d_bc, d_bc, H, H, H, self.num_rope_angles]

    def _compute_params(self, zxBCdtAtrap: torch.Tensor, batch_size: int, L=None):
        """Split the in_proj output and derive the per-step quantities
        (reference: src/models/mamba3.py:160-217).

        Returns z, x (…, H, P), B_exp, C_exp (…, R, H, D), ADT, DT, trap
        (…, H) and angle_raw (…, A), with … = (B,) or (B, L).
        """
        z, x, B_raw, C_raw, dd_dt, dd_A, trap_raw, angle_raw = torch.split(
            zxBCdtAtrap, self.split_sizes(), dim=-1)
        lead = zxBCdtAtrap.shape[:-1]
        R, G, H = self.mimo_rank, self.num_bc_heads, self.nheads
        z = z.reshape(*lead, H, self.headdim)
        x = x.reshape(*lead, H, self.headdim)
        B_raw = B_raw.reshape(*lead, R, G, self.d_state)
        C_raw = C_raw.reshape(*lead, R, G, self.d_state)

        # softplus(.) >= 0 > -A_floor, so the clamp always selects -A_floor
        # and A == +A_floor; kept as written for parity with the reference.
        A = -F.softplus(dd_A.float()).clamp(max=-self.A_floor)
        DT = F.softplus(dd_dt.float() + self.dt_bias)
        ADT = A * DT
        trap = torch.sigmoid(trap_raw.float())

        B_n = self.B_norm(B_raw.float())
        C_n = self.C_norm(C_raw.float())
        expand = (*lead, R, H, self.d_state)
        B_exp = B_n.expand(*expand) + self.B_bias.transpose(0, 1)
        C_exp = C_n.expand(*expand) + self.C_bias.transpose(0, 1)
        return z, x, B_exp, C_exp, ADT, DT, trap, angle_raw

    def _rope_bc(self, B_exp, C_exp, angles):
        """RoPE on the first split_tensor_size entries of B and C."""
        n = self.split_tensor_size
        ang = angles.unsqueeze(-3).expand(*angles.shape[:-2], self.mimo_rank, *angles.shape[-2:])
        B_proj = torch.cat([apply_rope(B_exp[..., :n], ang), B_exp[..., n:]], dim=-1)
        C_proj = torch.cat([apply_rope(C_exp[..., :n], ang), C_exp[..., n:]], dim=-1)
        return B_proj, C_proj

    def _ssm(self, x, B_proj, C_proj, ADT, DT, trap, h, bx_prev):
        if self.is_mimo:
            return mamba3_mimo_decode_ref(x, B_proj, C_proj, ADT, DT, trap, self.D,
                                          self.mimo_x, self.mimo_o, h, bx_prev)
        return mamba3_siso_decode_ref(x, B_proj[..., 0, :, :], C_proj[..., 0, :, :], ADT, DT,
                                      trap, self.D, h, bx_prev)

    # ------------------------------------------------------------------
    # decode
    # ------------------------------------------------------------------

    def step(self, u, angle_state, ssm_state, Bx_prev_state):
        """One autoregressive decode step in PyTorch (reference:
        src/models/mamba3.py:306-353).

        u (B, d_model); angle_state (B, H, A); ssm_state / Bx_prev_state
        (B, H, P, D) SISO or (B, H, D) MIMO.  Returns new tensors
        (out, angle_state, ssm_state, Bx_prev_state).
        """
        zx = self.in_proj(u)
        z, x, B_exp, C_exp, ADT, DT, trap, angle_raw = self._compute_params(zx, u.shape[0])
        angle_state = angle_state + angle_raw.float().unsqueeze(1) * DT.float().unsqueeze(-1)
        B_proj, C_proj = self._rope_bc(B_exp, C_exp, angle_state)
        y, ssm_state, Bx_prev_state = self._ssm(x, B_proj, C_proj, ADT, DT, trap,
                                                ssm_state, Bx_prev_state)
        y = (y * F.silu(z.float())).flatten(-2)
        return self.out_proj(y.to(u.dtype)), angle_state, ssm_state, Bx_prev_state

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        """Sequence forward (B, L, d_model) -> (B, L, d_model) by running the
        decode recurrence over L from a zero state (the reference's training
        path is the same sequential scan, src/models/mamba3.py:242-304)."""
        batch, L, _ = u.shape
        angle, h, bx = self.allocate_inference_cache(batch, device=u.device)
        outs = []
        for t in range(L):
            o, angle, h, bx = self.step(u[:, t], angle, h, bx)
            outs.append(o)
        return torch.stack(outs, dim=1)

    def allocate_inference_cache(self, batch_size: int, device=None, dtype=None):
        """Zero fp32 decode state (reference: src/models/mamba3.py:355-381):
        angle_state (B, H, A) and ssm_state / bx_prev of shape (B, H, D) for
        MIMO or (B, H, P, D) for SISO.  ``dtype`` is accepted and ignored:
        the state is always float32."""
        device = device or self.in_proj.weight.device
        H = self.nheads
        shape = (batch_size, H, self.d_state) if self.is_mimo else \
            (batch_size, H, self.headdim, self.d_state)
        z = lambda *s: torch.zeros(*s, device=device, dtype=torch.float32)  # noqa: E731
        return z(batch_size, H, self.num_rope_angles), z(*shape), z(*shape)

    def extra_repr(self) -> str:
        return (f"d_model={self.d_model}, d_state={self.d_state}, d_inner={self.d_inner}, "
                f"nheads={self.nheads}, headdim={self.headdim}, is_mimo={self.is_mimo}, "
                f"mimo_rank={self.mimo_rank}, num_rope_angles={self.num_rope_angles}")


class MambaBlock(nn.Module):
    """Residual block x + mixer(norm(x)) (reference: src/models/mamba3.py:412-421).
    The norm weight is created float32 regardless of the mixer's dtype, as in
    the reference."""

    def __init__(self, d_model: int, ssm_cfg: dict, device=None, dtype=None):
        super().__init__()
        self.norm = RMSNorm(d_model, device=device)
        self.mixer = Mamba3(d_model=d_model, **ssm_cfg, device=device, dtype=dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x + self.mixer(self.norm(x))


@dataclass
class MambaConfig:
    """Configuration of a stacked Mamba-3 language model; same fields and
    defaults as the reference (src/models/mamba3.py:396-409).  The attention,
    ``rms_norm``, ``residual_in_fp32`` and ``fused_add_norm`` fields are
    carried for interchange and, as in the reference, not acted on."""

    d_model: int = 2560
    d_intermediate: int = 0
    n_layer: int = 64
    vocab_size: int = 50277
    ssm_cfg: dict = field(default_factory=dict)
    attn_layer_idx: list = field(default_factory=list)
    attn_cfg: dict = field(default_factory=dict)
    rms_norm: bool = True
    residual_in_fp32: bool = True
    fused_add_norm: bool = True
    pad_vocab_size_multiple: int = 8
    tie_embeddings: bool = True


class MLP(nn.Module):
    """SwiGLU feed-forward layer (reference: src/models/mamba3.py:424-435)."""

    def __init__(self, d_model: int, d_intermediate: int, device=None, dtype=None):
        super().__init__()
        factory_kwargs = {"device": device, "dtype": dtype}
        self.fc1 = nn.Linear(d_model, 2 * d_intermediate, bias=False, **factory_kwargs)
        self.fc2 = nn.Linear(d_intermediate, d_model, bias=False, **factory_kwargs)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gate, val = self.fc1(x).chunk(2, dim=-1)
        return self.fc2(F.silu(gate) * val)


class MambaLMHeadModel(nn.Module):
    """Language model of stacked Mamba-3 blocks (reference:
    src/models/mamba3.py:438-481): embedding, ``n_layer`` residual blocks
    (each optionally followed by a residual SwiGLU MLP), final RMSNorm, LM
    head.  Parameters are created in the reference's order, so the same seed
    gives the same weights.  One deliberate difference: the reference
    declares ``lm_head = nn.Linear(vocab_size, d_model)``, whose weight has
    the transposed shape and works only when tied to the embedding; here it
    is ``nn.Linear(d_model, vocab_size)`` (the same number of random draws,
    and the same tied weight)."""

    def __init__(self, config: MambaConfig, device=None, dtype=None):
        factory_kwargs = {"device": device, "dtype": dtype}
        super().__init__()
        self.config = config
        vocab_size = config.vocab_size
        r = vocab_size % config.pad_vocab_size_multiple
        if r != 0:
            vocab_size += config.pad_vocab_size_multiple - r
        self.vocab_size = vocab_size
        self.embedding = nn.Embedding(vocab_size, config.d_model, **factory_kwargs)
        self.layers = nn.ModuleList([MambaBlock(config.d_model, config.ssm_cfg, **factory_kwargs)
                                     for _ in range(config.n_layer)])
        if config.d_intermediate > 0:
            self.mlp_norms = nn.ModuleList([RMSNorm(config.d_model, device=device) for _ in range(config.n_layer)])
            self.mlp_layers = nn.ModuleList([MLP(config.d_model, config.d_intermediate, **factory_kwargs)
                                             for _ in range(config.n_layer)])
        else:
            self.mlp_norms = None
            self.mlp_layers = None
        self.norm_f = RMSNorm(config.d_model, device=device)
        self.lm_head = nn.Linear(config.d_model, vocab_size, bias=False, **factory_kwargs)
        if config.tie_embeddings:
            self.lm_head.weight = self.embedding.weight

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        x = self.embedding(input_ids)
        for i, block in enumerate(self.layers):
            x = block(x)
            if self.mlp_layers is not None:
                x = x + self.mlp_layers[i](self.mlp_norms[i](x))
        x = self.norm_f(x)
        return self.lm_head(x)
