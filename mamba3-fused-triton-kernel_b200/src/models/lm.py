"""Token-by-token decoding of a ``MambaLMHeadModel``.

The reference has no decode path for its language model, only the
sequence ``forward`` (src/models/mamba3.py:473-481: embedding, blocks
``x + mixer(norm(x))`` each optionally followed by ``x + mlp(mlp_norm(x))``,
``norm_f``, ``lm_head``).  ``Mamba3LMDecoder.step`` computes the same thing
for one token per sequence with every mixer in its decode form:

    x = embedding(ids)
    xn = norm_0(x)
    for l:  o = mixer_l.step(xn)
            [MLP]  x, xm = x + o, mlp_norm_l(x + o);  x = x + mlp_l(xm)
            x, xn = x + o (or x), norm_{l+1}(x)      (norm_f after the last block)
    logits = lm_head(xn)

With a CUDA backend the residual add and the following norm are one kernel
(``m3_residual_rmsnorm``), every projection goes through
``src.kernels.linear.linear``, and ``warmup_cuda_graph`` captures the whole
token step -- embedding gather, all layers, the final norm and the LM head --
in one CUDA graph.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from src.kernels.linear import linear
from src.kernels.norm import residual_rmsnorm
from src.models.inference import Mamba3Decoder


class Mamba3LMDecoder:
    """Decoder over a ``MambaLMHeadModel``.  ``decoder_kwargs``: the
    ``Mamba3Decoder`` backend flags, applied to every layer;
    ``use_cuda_graph`` captures the whole token step."""

    def __init__(self, model, use_cuda_graph: bool = False, **decoder_kwargs):
        self.model = model
        self.blocks = list(model.layers)
        if not self.blocks:
            raise ValueError("model has no layers")
        self.layers = [Mamba3Decoder(b.mixer, **decoder_kwargs) for b in self.blocks]
        first = self.layers[0]
        self.cuda = first.use_triton or first.use_triton_fused or first.use_triton_full_fused or \
            first.use_compile or first.use_compile_cuda_graph
        self.use_cuda_graph = bool(use_cuda_graph) and self.cuda
        self._graph = None
        self._graph_ids = None
        self._graph_logits = None
        self._graph_states = None

    @property
    def vocab_size(self) -> int:
        return self.model.vocab_size

    def init_state(self, batch_size: int, device=None) -> list:
        """One ``{angle_state, ssm_state, bx_prev}`` dict per layer."""
        return [layer.init_state(batch_size, device=device) for layer in self.layers]

    def _norm_after(self, i: int):
        """The norm applied to the residual stream after block ``i``'s
        residual add: the next block's norm, or ``norm_f`` after the last."""
        return self.blocks[i + 1].norm if i + 1 < len(self.blocks) else self.model.norm_f

    def _step_eager(self, ids: torch.Tensor, states: list) -> torch.Tensor:
        m = self.model
        x = m.embedding(ids)
        mlp = m.mlp_layers
        if not self.cuda:
            xn = self.blocks[0].norm(x)
            for i, (layer, st) in enumerate(zip(self.layers, states)):
                o, _ = layer._step_pytorch(xn, st)
                x = x + o
                if mlp is not None:
                    x = x + mlp[i](m.mlp_norms[i](x))
                xn = self._norm_after(i)(x)
            return F.linear(xn, m.lm_head.weight)
        _, xn = residual_rmsnorm(x, None, self.blocks[0].norm.weight, self.blocks[0].norm.eps)
        for i, (layer, st) in enumerate(zip(self.layers, states)):
            o, _ = layer._graph_step_fn()(xn, st)
            if mlp is not None:
                x, xm = residual_rmsnorm(x, o, m.mlp_norms[i].weight, m.mlp_norms[i].eps)
                gate, val = linear(xm, mlp[i].fc1.weight).chunk(2, dim=-1)
                o = linear((F.silu(gate) * val).contiguous(), mlp[i].fc2.weight)
            nrm = self._norm_after(i)
            x, xn = residual_rmsnorm(x, o, nrm.weight, nrm.eps)
        return linear(xn, m.lm_head.weight)

    def warmup_cuda_graph(self, states: list, n_warmup: int = 3) -> None:
        """``n_warmup`` eager token steps (token id 0), then capture one token
        step in a CUDA graph that updates ``states`` in place."""
        if not self.use_cuda_graph:
            return
        h = states[0]["ssm_state"]
        self._graph_ids = torch.zeros(h.shape[0], dtype=torch.long, device=h.device)
        for _ in range(n_warmup):
            self._step_eager(self._graph_ids, states)
        torch.cuda.synchronize(h.device)
        self._graph = torch.cuda.CUDAGraph()
        self._graph_states = states
        with torch.cuda.graph(self._graph):
            self._graph_logits = self._step_eager(self._graph_ids, states)

    def step(self, input_ids: torch.Tensor, states: list) -> tuple:
        """One token per sequence: ``input_ids`` (batch,) -> (logits
        (batch, vocab), states)."""
        if self._graph is not None:
            if states is not self._graph_states:
                raise ValueError("a captured decoder steps the states it was captured with")
            self._graph_ids.copy_(input_ids)
            self._graph.replay()
            return self._graph_logits, states
        return self._step_eager(input_ids, states), states

    def decode_sequence(self, input_ids: torch.Tensor, states: list | None = None) -> tuple:
        """Feed ``input_ids`` (batch, length) token by token; returns
        (logits (batch, length, vocab), states) -- the reference ``forward``'s
        output, computed by the decode step."""
        B, L = input_ids.shape
        if states is None:
            states = self.init_state(B, device=input_ids.device)
        outs = []
        with torch.no_grad():
            for t in range(L):
                logits, states = self.step(input_ids[:, t], states)
                outs.append(logits.clone())
        return torch.stack(outs, dim=1), states
