"""Decoding a stack of residual Mamba-3 blocks.

A block is ``x + mixer(RMSNorm(x))`` (``MambaBlock``, src/models/mamba3.py:
412-421).  The reference decodes single layers only; a stacked model is
decoded by composing the layer step block by block:

    xn = RMSNorm_0(x)
    for l: o = mixer_l.step(xn);  x = x + o;  xn = RMSNorm_{l+1}(x)

With a CUDA backend the residual add and the next block's norm are one
kernel (``m3_residual_rmsnorm``), and ``warmup_cuda_graph`` captures the
whole stack -- every layer's projections, fused decode kernel and norm -- in
a single CUDA graph.
"""

from __future__ import annotations

import torch

from src.kernels.norm import residual_rmsnorm
from src.models.inference import Mamba3Decoder


class Mamba3StackDecoder:
    """``blocks``: a sequence of ``MambaBlock`` (``.norm``, ``.mixer``).
    ``decoder_kwargs``: the ``Mamba3Decoder`` backend flags, applied to every
    layer; ``use_cuda_graph`` captures the whole stack step."""

    def __init__(self, blocks, use_cuda_graph: bool = False, **decoder_kwargs):
        self.blocks = list(blocks)
        if not self.blocks:
            raise ValueError("empty stack")
        self.layers = [Mamba3Decoder(b.mixer, **decoder_kwargs) for b in self.blocks]
        first = self.layers[0]
        self.cuda = first.use_triton or first.use_triton_fused or first.use_triton_full_fused or \
            first.use_compile or first.use_compile_cuda_graph
        self.use_cuda_graph = bool(use_cuda_graph) and self.cuda
        self._graph = None
        self._graph_input = None
        self._graph_output = None
        self._graph_states = None

    @property
    def d_model(self) -> int:
        return self.blocks[0].mixer.d_model

    def init_state(self, batch_size: int, device=None) -> list:
        return [layer.init_state(batch_size, device=device) for layer in self.layers]

    def _layer_step(self, i: int):
        layer = self.layers[i]
        return layer._graph_step_fn() if self.cuda else layer._step_pytorch

    def _step_eager(self, x: torch.Tensor, states: list) -> tuple:
        n = len(self.blocks)
        if not self.cuda:
            for i, (blk, st) in enumerate(zip(self.blocks, states)):
                o, _ = self._layer_step(i)(blk.norm(x), st)
                x = x + o
            return x, states
        _, xn = residual_rmsnorm(x, None, self.blocks[0].norm.weight, self.blocks[0].norm.eps)
        for i, st in enumerate(states):
            o, _ = self._layer_step(i)(xn, st)
            nxt = self.blocks[i + 1].norm if i + 1 < n else None
            x, xn = residual_rmsnorm(x, o, None if nxt is None else nxt.weight,
                                     self.blocks[0].norm.eps if nxt is None else nxt.eps)
        return x, states

    def warmup_cuda_graph(self, states: list, n_warmup: int = 3) -> None:
        """``n_warmup`` eager stack steps on a zero input, then capture one
        whole stack step in a CUDA graph that updates ``states`` in place."""
        if not self.use_cuda_graph:
            return
        h = states[0]["ssm_state"]
        self._graph_input = torch.zeros(h.shape[0], self.d_model, device=h.device,
                                        dtype=self.blocks[0].mixer.in_proj.weight.dtype)
        for _ in range(n_warmup):
            self._step_eager(self._graph_input, states)
        torch.cuda.synchronize(h.device)
        self._graph = torch.cuda.CUDAGraph()
        self._graph_states = states
        with torch.cuda.graph(self._graph):
            self._graph_output, _ = self._step_eager(self._graph_input, states)

    def step(self, x: torch.Tensor, states: list) -> tuple:
        """One token through every block: x (batch, d_model) -> (x_out, states)."""
        if self._graph is not None:
            self._graph_input.copy_(x)
            self._graph.replay()
            return self._graph_output, self._graph_states
        return self._step_eager(x, states)
