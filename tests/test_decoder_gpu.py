"""Greedy decoding end to end: the B200 decoder (every op a libtrixium_b200 kernel, one CUDA graph
per token) against the oracle model (oracle/model.py, mirror.py:1002-1044 restated) on the same
synthetic image: the generated token ids must be identical.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PROMPT = [5, 17, 300, 42, 999, 0]


@pytest.fixture(scope="module")
def dec_mod():
    from trixium_b200 import decoder
    return decoder


def make(dec_mod, name, seed, max_pos=64):
    w = dec_mod.SyntheticWeights(dec_mod.CONFIGS[name], seed=seed)
    d = dec_mod.Decoder(w, max_pos=max_pos)
    return w, d


@pytest.mark.parametrize("name", ["tiny", "tiny-hybrid"])
def test_decoder_tokens_match_oracle(dec_mod, name):
    from oracle.model import OracleModel
    w, d = make(dec_mod, name, seed=3)
    orc = OracleModel(w, 64)
    if d.state:
        d.set_states(seed=9)
        orc.set_states({l: s.cpu().numpy() for l, s in d.state.items()})
    got = d.generate(PROMPT, 32)
    want = orc.generate(PROMPT, 32)
    assert got == want


@pytest.mark.parametrize("name", ["tiny", "tiny-hybrid"])
def test_decoder_graph_matches_eager(dec_mod, name):
    _, a = make(dec_mod, name, seed=4)
    _, b = make(dec_mod, name, seed=4)
    if a.state:
        a.set_states(seed=1)
        b.set_states(seed=1)
    eager = a.generate(PROMPT, 40)
    b.capture()
    graphed = b.generate(PROMPT, 40)
    assert eager == graphed
    assert int(b.pos.item()) == len(PROMPT) + 39
