"""Mamba-3 decoder with the sm_100a CUDA backends.

``Mamba3Decoder`` keeps the reference's constructor flags, ``init_state``,
``warmup_cuda_graph``, ``step`` and ``decode_sequence``
(src/models/inference.py:19-582).  Backends:

  use_triton_full_fused  in_proj -> ONE fused CUDA kernel -> out_proj
                         (the kernel updates ssm_state, bx_prev and
                         angle_state in place; small fp32 batches run both
                         projections on the library's small-batch GEMM).
                         In eager steps, layers the single-launch kernel
                         takes run the whole step -- both projections
                         included -- as ONE launch (``use_single_launch``,
                         default on) while the projections are small; a
                         captured step keeps the three launches, which
                         replay faster (single_launch_preferred).
  use_triton_fused       in_proj -> PyTorch split/norm/RoPE -> CUDA SSM+silu
                         kernel -> out_proj
  use_triton (default)   in_proj -> PyTorch split/norm/RoPE -> CUDA SSM
                         kernel -> silu -> out_proj
  use_triton=False       PyTorch reference decode (``Mamba3.step``)

The flag names are kept for drop-in compatibility; no Triton code exists in
this package.  Differences from the reference, all deliberate:

* A CUDA backend requested without a CUDA device raises instead of silently
  falling back to PyTorch, and so does a missing native library.
* ``use_compile`` / ``use_compile_cuda_graph`` are served by the fused CUDA
  kernel (eager / captured) instead of generating code with torch.compile.
* The two partially fused backends update ``angle_state`` in place, so the
  angle keeps accumulating under CUDA-graph replay (the reference rebinds it
  to a new tensor, which a captured graph never sees).
* The static graph input is allocated in the weight dtype, so bf16 models
  can be captured (the reference allocates it float32).
* The fused kernel reads bf16 in_proj output and bf16 parameters directly and
  writes its gated output in the weight dtype, fusing the reference's
  ``.float()`` and ``.to(u.dtype)`` casts.
* ``decode_sequence`` under graph replay keeps a copy of every step's output
  (the reference stacks the same static buffer seq_len times).
* ``use_single_launch`` (an extra keyword, default True) selects the
  single-launch step kernel for the full-fused backend where it applies.
* ``step_host`` (an extension) runs a step from and to pinned host memory.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from src import _native
from src.kernels import _launch
from src.kernels.linear import linear
from src.kernels.mimo_decode import mamba3_mimo_decode_triton
from src.kernels.mimo_decode_fused import mamba3_mimo_decode_fused_triton
from src.kernels.siso_decode import mamba3_siso_decode_triton
from src.kernels.siso_decode_fused import mamba3_siso_decode_fused_triton
from src.kernels.step import prepare_decode_step

# The single-launch step computes the projections on latency-oriented FP32
# FMA tiles; once they are large, the separate projection kernels win.  It
# serves eager steps of batches up to SINGLE_LAUNCH_MAX_BATCH whose projection
# work, 2 * B * d_model * (d_in_proj + d_inner) flop per step, stays within
# SINGLE_LAUNCH_MAX_FLOP for the weight dtype.
SINGLE_LAUNCH_MAX_BATCH = 256
SINGLE_LAUNCH_MAX_FLOP = {torch.float32: 3e8, torch.bfloat16: 1.5e8}
# step_host stores the single launch's output rows straight into pinned host
# memory for layers whose projection weights take at most this many bytes;
# larger layers replay the captured three launches and copy the output back.
# Measured on B200 (step_host, median us): MIMO R4 d256 (2.2 MB) batch 128
# 46.9 zero-copy against 48.1; d1024 fp32 (30 MB) batch 1 50.8 against 32.9.
STEP_HOST_SINGLE_MAX_WEIGHT_BYTES = 4 << 20


def single_launch_preferred(model, batch: int, graph: bool = False) -> bool:
    """Whether the decoder uses the single-launch step for this layer and
    batch (when the kernel takes the layer at all); ``graph``: for a step
    captured in a CUDA graph.  Only eager steps take it: there one launch
    saves the host time of two (19 against 59 us a step for the SISO d256
    layer on B200).  Replayed from a graph, the three launches measured
    faster on B200 for every layer tried: MIMO R4 d256 at batch 128 27.4
    against 32.2 us a step, d1024 fp32 at batch 1 22.7 against 49.3 us,
    SISO d256 18.9 against 24.6 us (the single launch's projection phases
    stream the weights on FFMA tiles, and its grid barriers wait for the
    slowest CTA)."""
    if graph:
        return False
    flop = 2.0 * batch * model.d_model * (model.d_in_proj + model.d_inner)
    limit = SINGLE_LAUNCH_MAX_FLOP.get(model.in_proj.weight.dtype, 0.0)
    return batch <= SINGLE_LAUNCH_MAX_BATCH and flop <= limit
from src.kernels.utils import apply_rope
from src.models.mamba3 import Mamba3


class Mamba3Decoder:
    """Autoregressive decoder around one ``Mamba3`` layer.

    Usage::

        decoder = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
        state = decoder.init_state(batch_size=8)
        decoder.warmup_cuda_graph(state)        # only with use_cuda_graph
        for u in token_embeddings:              # u: (batch, d_model)
            out, state = decoder.step(u, state)
    """

    def __init__(self, model: Mamba3, use_triton: bool = True, use_cuda_graph: bool = False,
                 use_compile: bool = False, use_triton_fused: bool = False,
                 use_compile_cuda_graph: bool = False, use_triton_full_fused: bool = False,
                 use_single_launch: bool = True):
        self.model = model
        # Flag resolution as in the reference (src/models/inference.py:52-57),
        # minus the silent CPU fallback.
        cuda_requested = use_triton or use_triton_fused or use_triton_full_fused or \
            use_compile or use_compile_cuda_graph
        if cuda_requested:
            _native.require_cuda_available()
            _native.load()  # fail loudly now if the library is missing
        self.use_triton = bool(use_triton)
        self.use_triton_fused = bool(use_triton_fused)
        self.use_triton_full_fused = bool(use_triton_full_fused)
        cuda_backend = self.use_triton or self.use_triton_fused or self.use_triton_full_fused
        self.use_cuda_graph = bool(use_cuda_graph) and cuda_backend
        self.use_compile = bool(use_compile) and not cuda_backend
        self.use_compile_cuda_graph = bool(use_compile_cuda_graph) and not self.use_cuda_graph
        if use_cuda_graph and not cuda_backend:
            print("Warning: CUDA Graph requires a CUDA backend, disabling")
        if use_compile and cuda_backend:
            print("Warning: use_compile is ignored when a CUDA backend is selected")

        self._cuda_graph = None
        self._graph_input = None
        self._graph_output = None
        self._graph_state = None
        self._fused_cache = None
        self._host_graph = None
        self._host_output = None
        self.use_single_launch = bool(use_single_launch)
        self._step_cache = None
        self._host_calls = 0

    # ------------------------------------------------------------------
    # public API
    # ------------------------------------------------------------------

    def init_state(self, batch_size: int, device=None, dtype=None) -> dict:
        """Zero decode state {angle_state, ssm_state, bx_prev} (float32)."""
        angle_state, ssm_state, bx_prev = self.model.allocate_inference_cache(
            batch_size, device=device, dtype=dtype)
        return {"angle_state": angle_state, "ssm_state": ssm_state, "bx_prev": bx_prev}

    def warmup_cuda_graph(self, state: dict, n_warmup: int = 10) -> None:
        """Run ``n_warmup`` eager steps on a zero input, then capture one
        whole decode step (in_proj, the CUDA kernel(s), out_proj) in a CUDA
        graph that updates ``state`` in place (reference:
        src/models/inference.py:97-160).  After this, ``step`` copies its
        input into a static buffer and replays the graph; the returned output
        tensor is the same static buffer every step."""
        if not (self.use_cuda_graph or self.use_compile_cuda_graph):
            return
        batch = state["ssm_state"].shape[0]
        device = state["ssm_state"].device
        self._graph_input = torch.zeros(batch, self.model.d_model, device=device,
                                        dtype=self.model.in_proj.weight.dtype)
        step_fn = self._graph_step_fn()
        for _ in range(n_warmup):
            step_fn(self._graph_input, state)
        torch.cuda.synchronize(device)
        self.check_device_error()
        self._cuda_graph = torch.cuda.CUDAGraph()
        self._host_graph = None
        self._host_output = None
        self._graph_state = state
        with torch.cuda.graph(self._cuda_graph):
            self._graph_output, self._graph_state = step_fn(self._graph_input, self._graph_state)

    def step_host(self, u_host: torch.Tensor) -> torch.Tensor:
        """One decode step from and to pinned host memory (an extension for
        serving loops whose token embeddings live on the host).

        ``u_host`` is a pinned (batch, d_model) tensor of the weight dtype.
        It is copied into the captured graph's input; where the
        single-launch kernel serves the layer and the projection weights are
        small (STEP_HOST_SINGLE_MAX_WEIGHT_BYTES), a second graph of that
        kernel writes the output rows straight into a pinned host buffer (no
        device-to-host copy), otherwise the captured step is replayed and its
        output copied back.  Returns the pinned output buffer once the
        device is idle: the same tensor every call, so copy it to keep a
        step's output.  Needs ``warmup_cuda_graph`` first; the state passed
        there is updated in place.  The first call validates and sets up;
        later calls only check shape and dtype, run on the current stream and
        wait with a device-wide synchronise, so call it with the decoder's
        device current (the usual one-GPU-per-process serving loop)."""
        if self._host_output is None:
            if self._cuda_graph is None:
                raise RuntimeError("step_host needs a captured graph: call warmup_cuda_graph first")
            dev = self._graph_input.device
            assert torch.cuda.current_device() == dev.index, "step_host needs the decoder's device current"
            assert u_host.device.type == "cpu" and u_host.is_pinned(), "u_host must be pinned host memory"
            self._host_output = torch.empty(self._graph_output.shape, dtype=self._graph_output.dtype,
                                            pin_memory=True)
            # the single launch as an eager step would take it: it stores the
            # output rows straight into host memory
            launch = None
            m = self.model
            wbytes = (m.in_proj.weight.numel() + m.out_proj.weight.numel()) * m.in_proj.weight.element_size()
            if self.use_single_launch and self._graph_step_fn() == self._step_triton_full_fused and \
                    wbytes <= STEP_HOST_SINGLE_MAX_WEIGHT_BYTES:
                launch = self._single_launch(self._graph_state, graph=False)
            if launch is not None and launch.accepts(self._graph_input):
                torch.cuda.synchronize(dev)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    launch.run(self._graph_input, self._host_output)  # kernel stores reach host memory
                self._host_graph = g
        gi = self._graph_input
        if u_host.shape != gi.shape or u_host.dtype != gi.dtype:
            raise AssertionError(f"u_host must be {tuple(gi.shape)} {gi.dtype}")
        gi.copy_(u_host, non_blocking=True)
        if self._host_graph is not None:
            self._host_graph.replay()
        else:
            self._cuda_graph.replay()
            self._host_output.copy_(self._graph_output, non_blocking=True)
        torch.cuda.synchronize()
        self._host_calls += 1
        if self._host_calls % self.DEVICE_ERROR_INTERVAL == 0:
            self.check_device_error()
        return self._host_output

    # step_host reads the library's device error word every this many calls
    # (the read costs a few small synchronous copies)
    DEVICE_ERROR_INTERVAL = 256

    def check_device_error(self) -> None:
        """Raise if a library kernel gave up a bounded wait since the last
        check (the word is process-wide and cleared by the read).

        Such a kernel skipped the rest of its work: the outputs and the state
        of the steps since the previous check are undefined, and the
        single-launch step's grid-barrier words no longer agree, so every
        later launch on its workspace would time out too.  Before raising,
        the workspace is zeroed again, so the decoder can go on after the
        caller has restored a state it trusts.  Synchronises the device.
        Called by ``warmup_cuda_graph``, every ``DEVICE_ERROR_INTERVAL``
        calls of ``step_host`` and at the end of ``decode_sequence``."""
        err = _native.device_error(reset=True)
        if err == 0:
            return
        launch = self._step_cache[1] if self._step_cache is not None else None
        if launch is not None:
            launch.workspace.zero_()
            torch.cuda.synchronize(launch.workspace.device)
        if err < 0:
            raise RuntimeError("the library's device error word could not be read")
        raise RuntimeError(f"a decode kernel gave up a bounded wait (device error {err:#x}): the outputs "
                           "and state of the steps since the last check are undefined; the step "
                           "workspace has been zeroed again")

    def step(self, u: torch.Tensor, state: dict) -> tuple:
        """One decode step: u (batch, d_model) -> (out (batch, d_model), state)."""
        if self._cuda_graph is not None:
            self._graph_input.copy_(u)
            self._cuda_graph.replay()
            return self._graph_output, self._graph_state
        if self.use_triton_full_fused or self.use_compile or self.use_compile_cuda_graph:
            return self._step_triton_full_fused(u, state)
        if self.use_triton_fused:
            return self._step_triton_fused(u, state)
        if self.use_triton:
            return self._step_triton(u, state)
        return self._step_pytorch(u, state)

    def decode_sequence(self, token_embeddings: torch.Tensor, state: dict = None) -> tuple:
        """Decode (batch, seq_len, d_model) step by step; returns
        (outputs (batch, seq_len, d_model), final state)."""
        batch, seq_len, _ = token_embeddings.shape
        if state is None:
            state = self.init_state(batch, device=token_embeddings.device)
        outs = []
        for t in range(seq_len):
            out, state = self.step(token_embeddings[:, t], state)
            # graph replay returns one static buffer; keep each step's value
            outs.append(out.clone() if self._cuda_graph is not None else out)
        if seq_len and token_embeddings.is_cuda and (self.use_triton or self.use_triton_fused
                                                     or self.use_triton_full_fused):
            self.check_device_error()
        return torch.stack(outs, dim=1), state

    # ------------------------------------------------------------------
    # backends
    # ------------------------------------------------------------------

    def _graph_step_fn(self):
        if self.use_triton_full_fused or self.use_compile_cuda_graph:
            return self._step_triton_full_fused
        if self.use_triton_fused:
            return self._step_triton_fused
        return self._step_triton

    def _step_pytorch(self, u: torch.Tensor, state: dict) -> tuple:
        """PyTorch reference decode (reference: src/models/inference.py:271-282)."""
        out, a, h, bx = self.model.step(u, state["angle_state"], state["ssm_state"],
                                        state["bx_prev"])
        state["angle_state"], state["ssm_state"], state["bx_prev"] = a, h, bx
        return out, state

    def _param_list(self):
        m = self.model
        return [m.dt_bias, m.D, m.B_norm.weight, m.C_norm.weight, m.B_bias, m.C_bias,
                m.mimo_x if m.is_mimo else None, m.mimo_o if m.is_mimo else None]

    def _fused_launch(self, state: dict):
        """Prepared fused launch for this state and the current parameters.

        Rebuilt when a parameter is replaced or modified in place (its
        ``_version`` changes) or another state is passed; otherwise reused,
        so an eager step costs one ctypes call for the kernel."""
        m = self.model
        params = self._param_list()
        key = (tuple(None if p is None else (p.data_ptr(), p._version, p.dtype) for p in params),
               tuple((t.data_ptr(), tuple(t.shape)) for t in
                     (state["ssm_state"], state["bx_prev"], state["angle_state"])))
        if self._fused_cache is not None and self._fused_cache[0] == key:
            return self._fused_cache[1]
        if not m.is_mimo:  # (H, 1, D) -> (H, D)
            params[4], params[5] = params[4][:, 0, :], params[5][:, 0, :]
        h = state["ssm_state"]
        launch = _launch.prepare_full_fused(
            m.is_mimo, h.shape[0], h.device, *params, h, state["bx_prev"], state["angle_state"],
            d_inner=m.d_inner, d_state=m.d_state, ngroups=m.num_bc_heads, mimo_rank=m.mimo_rank,
            nheads=m.nheads, headdim=m.headdim, split_tensor_size=m.split_tensor_size,
            num_rope_angles=m.num_rope_angles, A_floor=m.A_floor)
        self._fused_cache = (key, launch)
        return launch

    def _single_launch(self, state: dict, graph: bool = False):
        """Prepared single-launch step for this state and the current
        weights, or None where the kernel does not take the layer (or, with
        ``graph``, is not used in a captured step); rebuilt when a weight or
        parameter changes, another state is passed or the mode changes."""
        m = self.model
        ts = [m.in_proj.weight, m.out_proj.weight] + [p for p in self._param_list() if p is not None]
        key = (tuple((t.data_ptr(), t._version, t.dtype) for t in ts),
               tuple((t.data_ptr(), tuple(t.shape)) for t in
                     (state["ssm_state"], state["bx_prev"], state["angle_state"])), graph)
        if self._step_cache is None or self._step_cache[0] != key:
            use = single_launch_preferred(m, state["ssm_state"].shape[0], graph)
            self._step_cache = (key, prepare_decode_step(m, state) if use else None)
        return self._step_cache[1]

    def _step_triton_full_fused(self, u: torch.Tensor, state: dict) -> tuple:
        """in_proj -> fused CUDA step -> out_proj (reference:
        src/models/inference.py:476-559).  The kernel writes its gated output
        in the weight dtype, which is what out_proj consumes.  With
        ``use_single_launch`` the three run as one kernel where it applies."""
        m = self.model
        if self.use_single_launch:
            launch = self._single_launch(state, torch.cuda.is_current_stream_capturing())
            if launch is not None and launch.accepts(u):
                return launch.run(u), state
        zx = linear(u, m.in_proj.weight)
        if zx.dtype not in (torch.float32, torch.bfloat16) or zx.stride(1) != 1:
            zx = zx.float().contiguous()
        w_dtype = m.out_proj.weight.dtype
        y_dtype = w_dtype if w_dtype in (torch.float32, torch.bfloat16) else torch.float32
        y = torch.empty(u.shape[0], m.d_inner, device=u.device, dtype=y_dtype)
        self._fused_launch(state).run(zx, y)
        out = linear(y.to(u.dtype), m.out_proj.weight)
        return out, state

    def prefill(self, u: torch.Tensor, state: dict) -> tuple:
        """Feed a prompt: ``u`` (batch, length, d_model) -> (outputs (batch,
        length, d_model), state), the state advanced by all ``length`` tokens
        (what the reference computes with ``Mamba3.forward``'s sequential
        loop, src/models/mamba3.py:242-304, from a given state).  With the
        CUDA full-fused backend a layer runs one in_proj GEMM over all
        batch x length tokens, ONE prefill launch (MIMO: the streamed
        kernel's sequence form; SISO: one CTA per sequence and head with the
        head's state tile in registers; either way the carried state stays
        on chip from token to token) and one out_proj GEMM; shapes outside
        those kernels and other backends step token by token."""
        B, L = u.shape[0], u.shape[1]
        m = self.model
        if self.use_triton_full_fused and B > 0 and L > 0:
            flat = u.reshape(B * L, u.shape[2])
            zx = linear(flat, m.in_proj.weight)
            if zx.dtype not in (torch.float32, torch.bfloat16) or zx.stride(1) != 1:
                zx = zx.float().contiguous()
            w_dtype = m.out_proj.weight.dtype
            y_dtype = w_dtype if w_dtype in (torch.float32, torch.bfloat16) else torch.float32
            y = torch.empty(B * L, m.d_inner, device=u.device, dtype=y_dtype)
            if self._fused_launch(state).prefill(zx, y, L):
                out = linear(y.to(u.dtype), m.out_proj.weight)
                return out.view(B, L, -1), state
        outs = []
        for t in range(L):
            o, state = self.step(u[:, t].contiguous(), state)
            outs.append(o.clone())
        return torch.stack(outs, dim=1), state

    def _prep_projections(self, u: torch.Tensor, state: dict):
        """PyTorch split / norm / RoPE of the partially fused backends
        (reference: src/models/inference.py:305-358), with the angle state
        accumulated in place."""
        m = self.model
        zx = m.in_proj(u)
        z, x, B_exp, C_exp, ADT, DT, trap, angle_raw = m._compute_params(zx, u.shape[0])
        state["angle_state"].add_(angle_raw.float().unsqueeze(1) * DT.float().unsqueeze(-1))
        B_proj, C_proj = m._rope_bc(B_exp, C_exp, state["angle_state"])
        return z, x, B_proj, C_proj, ADT, DT, trap

    def _step_triton(self, u: torch.Tensor, state: dict) -> tuple:
        """PyTorch prep -> CUDA SSM kernel -> silu -> out_proj
        (reference: src/models/inference.py:294-383)."""
        m = self.model
        z, x, B_proj, C_proj, ADT, DT, trap = self._prep_projections(u, state)
        if m.is_mimo:
            y, _, _ = mamba3_mimo_decode_triton(x, B_proj, C_proj, ADT, DT, trap, m.D,
                                                m.mimo_x, m.mimo_o, state["ssm_state"],
                                                state["bx_prev"])
        else:
            y, _, _ = mamba3_siso_decode_triton(x, B_proj[:, 0], C_proj[:, 0], ADT, DT, trap, m.D,
                                                state["ssm_state"], state["bx_prev"])
        y = (y * F.silu(z.float())).flatten(1)
        return m.out_proj(y.to(u.dtype)), state

    def _step_triton_fused(self, u: torch.Tensor, state: dict) -> tuple:
        """PyTorch prep -> CUDA SSM+silu kernel -> out_proj
        (reference: src/models/inference.py:385-474)."""
        m = self.model
        z, x, B_proj, C_proj, ADT, DT, trap = self._prep_projections(u, state)
        if m.is_mimo:
            y, _, _ = mamba3_mimo_decode_fused_triton(x, B_proj, C_proj, ADT, DT, trap, m.D,
                                                      m.mimo_x, m.mimo_o, z.float(),
                                                      state["ssm_state"], state["bx_prev"])
        else:
            y, _, _ = mamba3_siso_decode_fused_triton(x, B_proj[:, 0], C_proj[:, 0], ADT, DT,
                                                      trap, m.D, z.float(), state["ssm_state"],
                                                      state["bx_prev"])
        return m.out_proj(y.flatten(1).to(u.dtype)), state
