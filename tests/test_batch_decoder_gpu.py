"""Batched greedy decoding (trixium_b200.decoder.BatchDecoder: the tensor-core rows projection, the
row-wise norms and SwiGLU, attention and DeltaNet over a sequence grid dimension) against the oracle
model (oracle/model.py, mirror.py:1002-1044 restated) run on each sequence alone: every sequence's
token ids must be identical, eagerly and replayed from a CUDA graph.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

PROMPTS = [[5, 17, 300, 42, 999, 0], [1, 2, 3, 4, 5, 6], [640, 12, 12, 7, 800, 33]]


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("name", ["tiny", "tiny-hybrid"])
def test_batch_decoder_tokens_match_oracle(name, graph):
    from oracle.model import OracleModel
    from trixium_b200 import decoder as D
    w = D.SyntheticWeights(D.CONFIGS[name], seed=5)
    bd = D.BatchDecoder(w, len(PROMPTS), max_pos=64)
    states = None
    if bd.state:
        one = D.Decoder(w, max_pos=64)
        one.set_states(seed=2)
        states = {l: s.clone() for l, s in one.state.items()}
        bd.set_states(states)
    if graph:
        bd.capture()
    got = bd.generate(PROMPTS, 24)
    for i, prompt in enumerate(PROMPTS):
        orc = OracleModel(w, 64)
        if states:
            orc.set_states({l: s.cpu().numpy() for l, s in states.items()})
        assert got[i] == orc.generate(prompt, 24), i


def test_batch_decoder_k_segments_match_decoder():
    """A K-segmented down projection (two ternary segments, trx_matvec_f_rows_kseg): every sequence's
    tokens equal the batch-1 decoder's (whose K-segment projection is pinned bit-exact to the
    reference's own segments), eagerly and replayed from a CUDA graph."""
    from trixium_b200 import decoder as D
    w = D.SyntheticWeights(D.CONFIGS["tiny-kseg"], seed=5)
    assert isinstance(w.layers[0]["down"], list) and len(w.layers[0]["down"]) == 2
    want = [D.Decoder(w, max_pos=64).generate(p, 24) for p in PROMPTS]
    for graph in (False, True):
        bd = D.BatchDecoder(w, len(PROMPTS), max_pos=64)
        if graph:
            bd.capture()
        assert bd.generate(PROMPTS, 24) == want, graph


def test_batch_decoder_rejects_k_segments():
    """More than two K-segments: refused."""
    from trixium_b200 import decoder as D
    cfg = D.CONFIGS["tiny"]
    w = D.SyntheticWeights(cfg, seed=1)
    w.layers[0]["down"] = [w.layers[0]["down"]] * 3
    with pytest.raises(ValueError):
        D.BatchDecoder(w, 2, max_pos=32)
    with pytest.raises(ValueError):
        D.BatchDecoder(D.SyntheticWeights(cfg, seed=1), 33, max_pos=32)
