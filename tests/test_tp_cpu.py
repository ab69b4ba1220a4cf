"""Tensor-parallel shard plan on the CPU: the plan covers every row (kv heads replicated when the
ranks outnumber them), the DeltaNet head renumbering keeps the kernel's tiled head map, and the
oracle model run sharded over gloo ranks (world size 2, and 4 with replicated kv heads) generates
the same tokens as the unsharded oracle model on the same image.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from trixium_b200 import decoder as D
from trixium_b200 import tp

PROMPT = [5, 17, 300, 42]


@pytest.mark.parametrize("name,world", [("tiny", 1), ("tiny", 2), ("tiny", 4), ("tiny-hybrid", 1),
                                        ("tiny-hybrid", 2), ("tiny-kv1", 2)])
def test_shard_plan_covers_rows(name, world):
    cfg = D.CONFIGS[name]
    for l in range(cfg.n_layer):
        if cfg.layer_type(l) == "d":
            shards = [tp.DeltaNetShard(cfg, r, world) for r in range(world)]
            ch = np.concatenate([s.channels for s in shards])
            assert sorted(ch) == list(range(cfg.dn_channels))
            assert sorted(np.concatenate([s.heads for s in shards])) == list(range(cfg.dn_nv))
            for s in shards:
                assert all(h % cfg.dn_nk - s.k0 == hl % s.nk for hl, h in enumerate(s.heads))
            assert [s.out0 for s in shards] == [r * cfg.dn_nv * cfg.dn_hv // world for r in range(world)]
        else:
            shards = [tp.AttnShard(cfg, r, world) for r in range(world)]
            assert sorted(np.concatenate([s.q_rows for s in shards])) == list(range(cfg.q_rows))
            g = max(1, world // cfg.n_kv)  # ranks per kv head (replicated when world > kv heads)
            assert sorted(np.concatenate([s.k_rows for s in shards])) == sorted(list(range(cfg.kv_rows)) * g)
            assert [s.head0 for s in shards] == [r * cfg.n_head // world for r in range(world)]
            rep = cfg.n_head // cfg.n_kv
            for s in shards:  # every query head sits with its own kv head
                assert s.head0 // rep == s.kv0 and (s.head0 + s.n_head - 1) // rep == s.kv1 - 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, name, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.tp_model import OracleTP
        full = D.SyntheticWeights(D.CONFIGS[name], seed=3, device="cpu")
        orc = OracleTP(tp.TPWeights(full, rank, world), max_pos=32)
        cfg = full.cfg
        states = {l: (np.random.default_rng(l).standard_normal((cfg.dn_nv, cfg.dn_hv, cfg.dn_hk)) /
                      np.sqrt(cfg.dn_hk)).astype(np.float32) for l in range(cfg.n_layer) if cfg.layer_type(l) == "d"}
        orc.set_states(states)
        out[rank] = orc.generate(PROMPT, 10)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("name,world", [("tiny", 2), ("tiny-hybrid", 2), ("tiny", 4), ("tiny-kv1", 2),
                                        ("tiny-hd256", 2)])
def test_sharded_oracle_matches_unsharded(name, world):
    """World 4 on "tiny" (2 kv heads): each kv head replicated on two ranks."""
    from oracle.model import OracleModel
    full = D.SyntheticWeights(D.CONFIGS[name], seed=3, device="cpu")
    cfg = full.cfg
    orc = OracleModel(full, 32)
    for l in range(cfg.n_layer):
        if cfg.layer_type(l) == "d":
            orc.layers[l]["S"][:] = (np.random.default_rng(l).standard_normal((cfg.dn_nv, cfg.dn_hv, cfg.dn_hk)) /
                                     np.sqrt(cfg.dn_hk)).astype(np.float32)
    want = orc.generate(PROMPT, 10)
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, name, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert all(out[r] == want for r in range(world))


@pytest.mark.parametrize("n_layer", [1, 2, 36])
def test_exchange_plan_signals_before_waits(n_layer):
    """Every gather point is signalled exactly once per step, by a launch that comes before the
    launch waiting on it, and every point is waited on (no rank can run ahead into a buffer that a
    peer has not read yet)."""
    plan = tp.exchange_plan(n_layer)
    signalled, waited = {}, set()
    for i, (op, l, sig, wt) in enumerate(plan):
        if wt is not None:
            assert wt in signalled and signalled[wt] < i, (op, l, wt)
            waited.add(wt)
        if sig is not None:
            assert sig not in signalled, (op, l, sig)
            signalled[sig] = i
    assert sorted(signalled) == list(range(4 * n_layer + 1))
    assert waited == set(signalled)
