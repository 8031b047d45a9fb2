"""Single-launch decode step of a MIMO or SISO layer.

``m3_mimo_step`` / ``m3_siso_step`` run in_proj, the full-step fused update
and out_proj of one decode step in ONE cooperative kernel (the three
launches of the reference's full-fused step, src/models/inference.py:
476-559, with the projections of src/models/mamba3.py:115,158).
``prepare_decode_step`` validates a layer and its state once and returns a
reusable launch, or ``None`` when the layer is outside the kernel's range
(MIMO heads not a multiple of 8, MIMO headdim or d_state > 128, mixed
dtypes, ...) and the three-launch path has to serve it.
"""

from __future__ import annotations

import torch

from src import _native as nat
from src.kernels._launch import check_state


def _uniform_dtype(tensors):
    dts = {t.dtype for t in tensors}
    if len(dts) != 1:
        return None
    dt = dts.pop()
    return dt if dt in (torch.float32, torch.bfloat16) else None


class DecodeStepLaunch:
    """A prepared single-launch step.  ``run(u, out)`` re-points the input
    and output rows and enqueues the kernel on the current stream of the
    state's device.  The caller keeps the model and the state alive while
    the object is used; the workspace belongs to the object (one per
    concurrently running step)."""

    __slots__ = ("dims", "args", "fn", "device", "dtype", "batch", "d_model", "keep", "workspace", "name")

    def __init__(self, dims, args, fn, device, dtype, batch, d_model, keep, workspace, name="m3_mimo_step"):
        self.dims, self.args, self.fn, self.device = dims, args, fn, device
        self.dtype, self.batch, self.d_model, self.keep, self.workspace = dtype, batch, d_model, keep, workspace
        self.name = name

    def accepts(self, u: torch.Tensor) -> bool:
        return (u.dtype == self.dtype and u.device == self.device and u.dim() == 2
                and tuple(u.shape) == (self.batch, self.d_model) and u.stride(1) == 1
                and u.stride(0) % 4 == 0 and u.data_ptr() % 16 == 0)

    def run(self, u: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        assert self.accepts(u), "input must be a (batch, d_model) row-major tensor of the layer's dtype"
        if out is None:
            out = torch.empty(self.batch, self.d_model, device=self.device, dtype=self.dtype)
        assert out.dtype == self.dtype and tuple(out.shape) == (self.batch, self.d_model) and out.stride(1) == 1
        a = self.args
        a.u = u.data_ptr(); a.u_stride_b = u.stride(0)
        a.out = out.data_ptr(); a.out_stride_b = out.stride(0)
        with nat.device_guard(self.device):
            st = self.fn(self.dims, a, nat.stream_handle(self.device))
        nat.check(st, self.name)
        return out


def prepare_decode_step(model, state: dict):
    """A ``DecodeStepLaunch`` for ``model`` (a ``Mamba3``) and ``state``, or
    ``None`` if the single-launch kernel does not take this layer."""
    m = model
    h = state["ssm_state"]
    if not h.is_cuda or m.num_bc_heads != 1:
        return None
    W_in, W_out = m.in_proj.weight, m.out_proj.weight
    params = [m.dt_bias, m.D, m.B_norm.weight, m.C_norm.weight, m.B_bias, m.C_bias]
    if m.is_mimo:
        params += [m.mimo_x, m.mimo_o]
    dtype = _uniform_dtype([W_in, W_out] + params)
    if dtype is None or any(t.device != h.device for t in [W_in, W_out] + params):
        return None
    if W_in.stride(1) != 1 or W_out.stride(1) != 1 or not all(t.is_contiguous() for t in params):
        return None
    B = h.shape[0]
    check_state("ssm_state", h)
    check_state("bx_prev", state["bx_prev"])
    check_state("angle_state", state["angle_state"])
    dims = nat.Dims(batch=B, nheads=m.nheads, headdim=m.headdim, d_state=m.d_state,
                    mimo_rank=m.mimo_rank, num_rope_angles=m.num_rope_angles, ngroups=1,
                    d_inner=m.d_inner, A_floor=float(m.A_floor))
    code = nat.M3_BF16 if dtype == torch.bfloat16 else nat.M3_F32
    lib = nat.load()
    kind = "mimo" if m.is_mimo else "siso"
    nbytes = getattr(lib, f"m3_{kind}_step_workspace_bytes")(dims, m.d_model, code)
    if nbytes < 0:
        if -nbytes == nat.M3_ERR_UNSUPPORTED:
            return None
        nat.check(int(-nbytes), f"m3_{kind}_step_workspace_bytes")
    workspace = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=h.device)
    a = nat.StepArgs()
    a.d_model, a.dtype = m.d_model, code
    a.in_proj_w, a.in_proj_stride = W_in.data_ptr(), W_in.stride(0)
    a.out_proj_w, a.out_proj_stride = W_out.data_ptr(), W_out.stride(0)
    a.dt_bias, a.D, a.B_norm_w, a.C_norm_w = (t.data_ptr() for t in params[:4])
    a.B_bias, a.C_bias = params[4].data_ptr(), params[5].data_ptr()
    a.mimo_x, a.mimo_o = (params[6].data_ptr(), params[7].data_ptr()) if m.is_mimo else (None, None)
    a.ssm_state, a.bx_prev, a.angle_state = (h.data_ptr(), state["bx_prev"].data_ptr(),
                                             state["angle_state"].data_ptr())
    a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    # alignment of the weights and biases is checked by the library at run()
    return DecodeStepLaunch(dims, a, getattr(lib, f"m3_{kind}_step"), h.device, dtype, B, m.d_model,
                            [W_in, W_out, *params, h, state["bx_prev"], state["angle_state"]], workspace,
                            f"m3_{kind}_step")


def decode_step(model, u: torch.Tensor, state: dict) -> torch.Tensor:
    """One decode step of ``model`` through the single-launch kernel (the
    state is updated in place); raises if the layer is outside its range."""
    launch = prepare_decode_step(model, state)
    if launch is None:
        raise ValueError("this layer is outside the single-launch step kernel's range")
    return launch.run(u)
