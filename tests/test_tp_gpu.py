"""The tensor-parallel decoder (trixium_b200.tp) against the single-GPU decoder on the same synthetic
image: identical greedy tokens.  World size 1 always; world size 2 (two NCCL ranks, one GPU each)
when the box has two GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

PROMPT = [5, 17, 300, 42, 999]
N_NEW = 24


def single_gpu_tokens(name, device=0):
    from trixium_b200 import decoder as D, ops
    torch.cuda.set_device(device)
    w = D.SyntheticWeights(D.CONFIGS[name], seed=5)
    d = D.Decoder(w, ctx=ops.Context(device), max_pos=64)
    if d.state:
        d.set_states(seed=2)
    return d.generate(PROMPT, N_NEW)


def tp_tokens(name, rank, world, group=None, graph=False, p2p=False):
    from trixium_b200 import decoder as D, ops, tp
    full = D.SyntheticWeights(D.CONFIGS[name], seed=5)
    dec = tp.TPDecoder(tp.TPWeights(full, rank, world), group=group, ctx=ops.Context(torch.cuda.current_device()),
                       max_pos=64, p2p=p2p)
    assert dec.p2p == (p2p and world > 1)
    del full
    if dec.state:
        dec.set_states(seed=2)
    if graph:
        dec.capture()
    toks = dec.generate(PROMPT, N_NEW)
    dec.release()
    return toks


@pytest.mark.parametrize("name", ["tiny", "tiny-hybrid"])
def test_tp_world1_matches_decoder(name):
    want = single_gpu_tokens(name)
    assert tp_tokens(name, 0, 1) == want
    assert tp_tokens(name, 0, 1, graph=True) == want


def _rank(rank, world, port, name, out, p2p=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    torch.cuda.set_device(rank)
    from datetime import timedelta
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                         device_id=torch.device("cuda", rank))
    try:
        out[rank] = (tp_tokens(name, rank, world, graph=False, p2p=p2p),
                     tp_tokens(name, rank, world, graph=True, p2p=p2p))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", ["tiny", "tiny-hybrid", "tiny-kv1", "tiny-kseg", "tiny-hd256"])
def test_tp_world2_matches_decoder(name):
    """tiny-kv1 has one kv head: both ranks hold it (replicated) and split its query heads."""
    want = single_gpu_tokens(name)
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank, args=(r, 2, port, name, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    for r in range(2):
        assert out[r][0] == want and out[r][1] == want


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", ["tiny", "tiny-kv1", "tiny-hybrid", "tiny-kseg", "tiny-hd256"])
def test_tp_world2_peer_exchange_matches_decoder(name):
    """The all-gathers done by the kernels themselves over peer memory (tagged words, no NCCL on the
    data path)."""
    want = single_gpu_tokens(name)
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank, args=(r, 2, port, name, out, True)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    for r in range(2):
        assert out[r][0] == want and out[r][1] == want
