"""Tensor -> C-ABI marshalling for the decode entry points.

Every public kernel function in this package ends up here: it checks shapes
the way the reference launchers do, brings auxiliary inputs to a supported
dtype, fills the ctypes argument block of include/mamba3_b200.h and calls the
library on the current CUDA stream of the state's device.
"""

from __future__ import annotations

import torch

from src import _native as nat

_IO_DTYPES = (torch.float32, torch.bfloat16)


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.float32 else t.float()


def _io(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype in _IO_DTYPES else t.float()


def check_state(name: str, t: torch.Tensor) -> None:
    assert t.is_cuda, f"{name} must be a CUDA tensor"
    assert t.dtype == torch.float32, f"{name} must be float32 (got {t.dtype})"
    assert t.is_contiguous(), f"{name} must be contiguous: it is updated in place"


def _same_device(dev: torch.device, *ts) -> None:
    for t in ts:
        if t is not None:
            assert t.device == dev, f"all tensors must be on {dev} (got {t.device})"


def ssm_decode(mimo: bool, x, B_proj, C_proj, ADT, DT, trap, D_skip, h, bx_prev,
               mimo_x=None, mimo_o=None, z=None) -> torch.Tensor:
    """One state-update-only step (gated by silu(z) when ``z`` is given).

    Updates ``h`` and ``bx_prev`` in place and returns ``y`` with the shape
    and dtype of ``x`` (the reference allocates ``torch.empty_like(x)``).
    """
    y = torch.empty_like(x)
    Bsz, H, P = x.shape
    if Bsz == 0:
        return y
    dev = h.device
    check_state("h", h)
    check_state("bx_prev", bx_prev)
    _same_device(dev, x, B_proj, C_proj, ADT, DT, trap, D_skip, bx_prev, mimo_x, mimo_o, z)
    D = B_proj.shape[-1]
    R = B_proj.shape[1] if mimo else 1
    # every input is read at the indices its shape implies: check them all
    bc_shape = (Bsz, R, H, D) if mimo else (Bsz, H, D)
    assert tuple(B_proj.shape) == bc_shape, f"B_proj must be {bc_shape}, got {tuple(B_proj.shape)}"
    assert tuple(C_proj.shape) == bc_shape, f"C_proj must be {bc_shape}, got {tuple(C_proj.shape)}"
    for name, t in (("ADT", ADT), ("DT", DT), ("trap", trap)):
        assert tuple(t.shape) == (Bsz, H), f"{name} must be {(Bsz, H)}, got {tuple(t.shape)}"
    assert tuple(D_skip.shape) == (H,), f"D_skip must be {(H,)}, got {tuple(D_skip.shape)}"
    if z is not None:
        assert tuple(z.shape) == (Bsz, H, P), f"z must be {(Bsz, H, P)}, got {tuple(z.shape)}"
    if mimo:
        for name, t in (("mimo_x", mimo_x), ("mimo_o", mimo_o)):
            assert tuple(t.shape) == (H, R, P), f"{name} must be {(H, R, P)}, got {tuple(t.shape)}"

    xx = _io(x)
    yy = y if y.dtype in _IO_DTYPES else torch.empty_like(x, dtype=torch.float32)
    Bp, Cp = _f32(B_proj), _f32(C_proj)
    adt, dt, tr, dsk = _f32(ADT), _f32(DT), _f32(trap), _f32(D_skip)

    dims = nat.Dims(batch=Bsz, nheads=H, headdim=P, d_state=D, mimo_rank=R,
                    num_rope_angles=0, ngroups=1, d_inner=H * P, A_floor=0.0)
    a = nat.SsmArgs()
    a.x = xx.data_ptr(); a.x_sb, a.x_sh, a.x_sp = xx.stride(); a.x_dtype = nat.dtype_code(xx)
    a.y = yy.data_ptr(); a.y_sb, a.y_sh, a.y_sp = yy.stride(); a.y_dtype = nat.dtype_code(yy)
    if z is not None:
        zz = _io(z)
        a.z = zz.data_ptr(); a.z_sb, a.z_sh, a.z_sp = zz.stride(); a.z_dtype = nat.dtype_code(zz)
    a.B_proj, a.C_proj = Bp.data_ptr(), Cp.data_ptr()
    if mimo:
        a.B_sb, a.B_sr, a.B_sh, a.B_sd = Bp.stride()
        a.C_sb, a.C_sr, a.C_sh, a.C_sd = Cp.stride()
    else:
        a.B_sb, a.B_sh, a.B_sd = Bp.stride()
        a.C_sb, a.C_sh, a.C_sd = Cp.stride()
    a.ADT = adt.data_ptr(); a.adt_sb, a.adt_sh = adt.stride()
    a.DT = dt.data_ptr(); a.dt_sb, a.dt_sh = dt.stride()
    a.trap = tr.data_ptr(); a.trap_sb, a.trap_sh = tr.stride()
    a.D_skip = dsk.data_ptr(); a.D_sh = dsk.stride(0)
    if mimo:
        mx, mo = _f32(mimo_x), _f32(mimo_o)
        a.mimo_x = mx.data_ptr(); a.mx_sh, a.mx_sr, a.mx_sp = mx.stride()
        a.mimo_o = mo.data_ptr(); a.mo_sh, a.mo_sr, a.mo_sp = mo.stride()
    a.h, a.bx_prev = h.data_ptr(), bx_prev.data_ptr()

    lib = nat.load()
    if mimo:
        fn = lib.m3_mimo_decode_fused if z is not None else lib.m3_mimo_decode
    else:
        fn = lib.m3_siso_decode_fused if z is not None else lib.m3_siso_decode
    with nat.device_guard(dev):
        st = fn(dims, a, nat.stream_handle(dev))
    nat.check(st, fn.__name__)
    if yy is not y:
        y.copy_(yy)
    return y


def _param_set(tensors):
    """Bring the per-head parameters to one dtype the kernel reads (all f32
    or all bf16) and contiguous layout."""
    present = [t for t in tensors if t is not None]
    if all(t.dtype == torch.bfloat16 for t in present):
        code = nat.M3_BF16
        out = [None if t is None else t.contiguous() for t in tensors]
    else:
        code = nat.M3_F32
        out = [None if t is None else _f32(t).contiguous() for t in tensors]
    return code, out


class FullFusedLaunch:
    """A full-fused launch whose arguments are marshalled once.

    ``run(zx, y)`` re-points the in_proj output and the output buffer (both
    may change between steps) and enqueues the kernel on the current stream
    of the state's device: one ctypes call, no re-validation of the
    unchanged state and parameters.  The caller keeps every tensor passed to
    ``prepare_full_fused`` alive while the object is used.
    """

    __slots__ = ("dims", "args", "fn", "device", "keep", "zx_dtype", "y_dtype", "batch", "d_in_proj", "d_inner")

    def __init__(self, dims, args, fn, device, keep, batch, d_in_proj, d_inner):
        self.dims, self.args, self.fn, self.device, self.keep = dims, args, fn, device, keep
        self.batch, self.d_in_proj, self.d_inner = batch, d_in_proj, d_inner

    def run(self, zx: torch.Tensor, y: torch.Tensor) -> None:
        assert zx.shape == (self.batch, self.d_in_proj) and zx.stride(1) == 1 and zx.device == self.device
        assert y.shape == (self.batch, self.d_inner) and y.stride(1) == 1 and y.device == self.device
        a = self.args
        a.zx = zx.data_ptr(); a.zx_stride_b = zx.stride(0); a.zx_dtype = nat.dtype_code(zx)
        a.y = y.data_ptr(); a.y_stride_b = y.stride(0); a.y_dtype = nat.dtype_code(y)
        with nat.device_guard(self.device):
            st = self.fn(self.dims, a, nat.stream_handle(self.device))
        nat.check(st, self.fn.__name__)

    def prefill(self, zx: torch.Tensor, y: torch.Tensor, seq_len: int) -> bool:
        """Prefill (``m3_mimo_prefill`` / ``m3_siso_prefill``): ``zx`` / ``y``
        hold batch x seq_len rows (row b * seq_len + t); the state is
        stepped through all tokens in one launch.  False (nothing enqueued)
        when the layer's shape is outside the prefill kernel's range."""
        n = self.batch * seq_len
        assert zx.shape == (n, self.d_in_proj) and zx.stride(1) == 1 and zx.device == self.device
        assert y.shape == (n, self.d_inner) and y.stride(1) == 1 and y.device == self.device
        a = self.args
        a.zx = zx.data_ptr(); a.zx_stride_b = zx.stride(0); a.zx_dtype = nat.dtype_code(zx)
        a.y = y.data_ptr(); a.y_stride_b = y.stride(0); a.y_dtype = nat.dtype_code(y)
        lib = nat.load()
        fn = lib.m3_mimo_prefill if self.fn.__name__.startswith("m3_mimo") else lib.m3_siso_prefill
        with nat.device_guard(self.device):
            st = fn(self.dims, a, seq_len, nat.stream_handle(self.device))
        if st == nat.M3_ERR_UNSUPPORTED:
            return False
        nat.check(st, fn.__name__)
        return True


def prepare_full_fused(mimo: bool, batch: int, device, dt_bias, D_skip, B_norm_w, C_norm_w, B_bias,
                       C_bias, mimo_x, mimo_o, h, bx_prev, angle_state, *, d_inner, d_state, ngroups,
                       mimo_rank, nheads, headdim, split_tensor_size, num_rope_angles,
                       A_floor) -> FullFusedLaunch:
    """Validate the state and parameters once and return a reusable launch."""
    Bsz = batch
    H, P, D = nheads, headdim, d_state
    R = mimo_rank if mimo else 1
    dev = h.device
    assert h.is_cuda
    check_state("ssm_state", h)
    check_state("bx_prev", bx_prev)
    check_state("angle_state", angle_state)
    assert split_tensor_size == 2 * num_rope_angles, "split_tensor_size must be 2 * num_rope_angles"
    assert d_inner == H * P, "d_inner must equal nheads * headdim"
    if mimo and R not in nat.SUPPORTED_RANKS:
        raise ValueError(f"Unsupported mimo_rank={R}. Supported values: {list(nat.SUPPORTED_RANKS)}")
    d_in_proj = 2 * d_inner + 2 * D * ngroups * R + 3 * H + num_rope_angles
    _same_device(dev, bx_prev, angle_state)
    shapes = [("dt_bias", dt_bias, (H,)), ("D", D_skip, (H,)), ("B_norm_weight", B_norm_w, (D,)),
              ("C_norm_weight", C_norm_w, (D,)),
              ("B_bias", B_bias, (H, R, D) if mimo else (H, D)),
              ("C_bias", C_bias, (H, R, D) if mimo else (H, D))]
    if mimo:
        shapes += [("mimo_x", mimo_x, (H, R, P)), ("mimo_o", mimo_o, (H, R, P))]
    for name, t, shp in shapes:
        assert tuple(t.shape) == shp, f"{name} must be {shp}, got {tuple(t.shape)}"
        _same_device(dev, t)
    assert tuple(angle_state.shape) == (Bsz, H, num_rope_angles)
    assert tuple(h.shape) == tuple(bx_prev.shape) == ((Bsz, H, D) if mimo else (Bsz, H, P, D))
    code, keep = _param_set([dt_bias, D_skip, B_norm_w, C_norm_w, B_bias, C_bias,
                             mimo_x if mimo else None, mimo_o if mimo else None])
    dtb, dsk, wb, wc, bb, bc, mx, mo = keep
    dims = nat.Dims(batch=Bsz, nheads=H, headdim=P, d_state=D, mimo_rank=R,
                    num_rope_angles=num_rope_angles, ngroups=ngroups, d_inner=d_inner,
                    A_floor=float(A_floor))
    a = nat.FullArgs()
    a.param_dtype = code
    a.dt_bias, a.D, a.B_norm_w, a.C_norm_w = dtb.data_ptr(), dsk.data_ptr(), wb.data_ptr(), wc.data_ptr()
    a.B_bias, a.C_bias = bb.data_ptr(), bc.data_ptr()
    if mimo:
        a.mimo_x, a.mimo_o = mx.data_ptr(), mo.data_ptr()
    a.ssm_state, a.bx_prev, a.angle_state = h.data_ptr(), bx_prev.data_ptr(), angle_state.data_ptr()
    lib = nat.load()
    fn = lib.m3_mimo_full_fused if mimo else lib.m3_siso_full_fused
    return FullFusedLaunch(dims, a, fn, dev, keep + [h, bx_prev, angle_state], Bsz, d_in_proj, d_inner)


def full_fused(mimo: bool, zx, dt_bias, D_skip, B_norm_w, C_norm_w, B_bias, C_bias,
               mimo_x, mimo_o, h, bx_prev, angle_state, *, d_inner, d_state, ngroups,
               mimo_rank, nheads, headdim, split_tensor_size, num_rope_angles, A_floor,
               y: torch.Tensor | None = None) -> torch.Tensor:
    """One full decode step between in_proj and out_proj.

    Updates ``h``, ``bx_prev`` and ``angle_state`` in place.  Writes the
    gated output into ``y`` ((B, H*P) rows, f32 or bf16) when given, else
    into a new (B, H, P) float32 tensor, and returns it.
    """
    Bsz = zx.shape[0]
    H, P = nheads, headdim
    if y is None:
        y = torch.empty(Bsz, H, P, device=zx.device, dtype=torch.float32)
    if Bsz == 0:
        return y
    assert zx.is_cuda and h.is_cuda
    if mimo and mimo_rank not in nat.SUPPORTED_RANKS:
        raise ValueError(f"Unsupported mimo_rank={mimo_rank}. "
                         f"Supported values: {list(nat.SUPPORTED_RANKS)}")
    launch = prepare_full_fused(
        mimo, Bsz, h.device, dt_bias, D_skip, B_norm_w, C_norm_w, B_bias, C_bias, mimo_x, mimo_o,
        h, bx_prev, angle_state, d_inner=d_inner, d_state=d_state, ngroups=ngroups,
        mimo_rank=mimo_rank, nheads=nheads, headdim=headdim, split_tensor_size=split_tensor_size,
        num_rope_angles=num_rope_angles, A_floor=A_floor)
    assert zx.dim() == 2 and zx.shape[1] == launch.d_in_proj, \
        f"zxBCdtAtrap must be (B, {launch.d_in_proj}); got {tuple(zx.shape)}"
    _same_device(h.device, zx, y)
    zz = _io(zx)
    if zz.stride(1) != 1:
        zz = zz.contiguous()
    y2 = y.view(Bsz, -1) if y.dim() == 3 else y
    launch.run(zz, y2)
    return y
