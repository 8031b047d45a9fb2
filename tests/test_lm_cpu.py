"""Language model (src/models/mamba3.py MambaLMHeadModel, src/models/lm.py
Mamba3LMDecoder) against fixtures made by running the reference's own
MambaLMHeadModel (tests/golden/make_golden.py): the same seed gives the same
weights, ``forward`` gives the reference's logits, and decoding the
sequence token by token (PyTorch decode path) gives them too."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from src.models.lm import Mamba3LMDecoder
from src.models.mamba3 import MambaConfig, MambaLMHeadModel


def _model(g):
    torch.manual_seed(g["meta"]["seed"])
    return MambaLMHeadModel(MambaConfig(**g["meta"]["config"])).eval()


@pytest.mark.parametrize("name", golden_names("lm"))
def test_same_weights_and_forward(name):
    g = load_golden(name)
    model = _model(g)
    for pname, prm in model.state_dict().items():
        want = float(g["sum." + pname])
        got = float(prm.detach().double().sum())
        assert abs(got - want) <= 1e-9 * max(1.0, abs(want)) * prm.numel(), pname
    assert model.lm_head.weight is model.embedding.weight
    with torch.no_grad():
        logits = model(torch.from_numpy(g["input_ids"]))
    np.testing.assert_allclose(logits.numpy(), g["logits"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", golden_names("lm"))
def test_token_by_token_decode(name):
    g = load_golden(name)
    model = _model(g)
    dec = Mamba3LMDecoder(model, use_triton=False)
    logits, states = dec.decode_sequence(torch.from_numpy(g["input_ids"]))
    assert logits.shape == g["logits"].shape and len(states) == g["meta"]["config"]["n_layer"]
    np.testing.assert_allclose(logits.numpy(), g["logits"], rtol=1e-5, atol=1e-5)


def test_vocab_padding_and_untied_head():
    cfg = MambaConfig(d_model=32, n_layer=1, vocab_size=13, tie_embeddings=False,
                      ssm_cfg=dict(d_state=16, headdim=16))
    m = MambaLMHeadModel(cfg)
    assert m.vocab_size == 16 and m.lm_head.weight.shape == (16, 32)
    assert m(torch.zeros(1, 2, dtype=torch.long)).shape == (1, 2, 16)
