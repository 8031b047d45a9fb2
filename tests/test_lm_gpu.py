"""The language-model decoder on the CUDA decode path (fused kernels, the
residual-norm kernel, the library's projections), eager and captured in
one CUDA graph, against the reference's logits (fixtures made by running
its MambaLMHeadModel.forward)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from src.models.lm import Mamba3LMDecoder
from src.models.mamba3 import MambaConfig, MambaLMHeadModel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("name", golden_names("lm"))
def test_cuda_decode_matches_reference(name, graph):
    g = load_golden(name)
    torch.manual_seed(g["meta"]["seed"])
    model = MambaLMHeadModel(MambaConfig(**g["meta"]["config"])).cuda().eval()
    dec = Mamba3LMDecoder(model, use_triton_full_fused=True, use_cuda_graph=graph)
    ids = torch.from_numpy(g["input_ids"]).cuda()
    states = dec.init_state(ids.shape[0], device="cuda")
    if graph:
        dec.warmup_cuda_graph(states, n_warmup=0)
        assert dec._graph is not None
    logits, _ = dec.decode_sequence(ids, states)
    np.testing.assert_allclose(logits.cpu().numpy(), g["logits"], rtol=1e-4, atol=1e-4)
