"""Decode attention (trx_attn_decode) and the gated-DeltaNet step (trx_deltanet_step), through the
C ABI, replayed position by position against the reference's own firmware mirror: the traced layer
outputs of model/mirror.py hybrid27_generate (exact=True, mathematical profile) on a reference-written
hybrid image whose output projections are identities (tests/golden/mirror_layers_*.npz, made by
tests/golden/make_golden.py hybrid_kernel_case).  The kernels keep an fp16 KV cache where the mirror
keeps fp32, and sum in parallel where the mirror sums in sequence: every step's output is within
1e-3 of its scale (max |got - want| / max(1, max |want|)).
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(scope="module")
def ops():
    from trixium_b200 import ops as o
    return o


@pytest.fixture(scope="module")
def ctx(ops):
    c = ops.Context(0)
    yield c
    c.close()


def _err(got, want):
    return float(np.abs(got.cpu().numpy().astype(np.float64) - want).max() / max(1.0, float(np.abs(want).max())))


@pytest.mark.parametrize("kv", ["fp16", "fp32"])
@pytest.mark.parametrize("name", ["hd64", "hd256"])
def test_attention_matches_the_mirror(ops, ctx, name, kv):
    """fp16 cache (the build's): 1e-3 of the output scale; fp32 cache (the mirror's own,
    trx_attn_decode_f32cache): 2e-5."""
    d = load(os.path.join(GOLDEN, f"mirror_layers_{name}.npz"))
    H, Hkv, hd, npos = int(d["n_head"]), int(d["n_kv"]), int(d["head_dim"]), int(d["npos"])
    dv = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    shape = ops.attn_shape(H, Hkv, hd, npos, rope_dims=int(d["rope_dims"]), gated=bool(d["gated"]),
                           eps=float(d["eps"]))
    freq = dv(d["rope_freq"])
    n = 0
    for l, dn in enumerate(d["layer_types"]):
        if dn:
            continue
        kc = torch.zeros(npos, Hkv, hd, dtype=torch.float16 if kv == "fp16" else torch.float32, device="cuda")
        vc = torch.zeros_like(kc)
        pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        qn, kn = dv(d[f"l{l}_q_norm"]), dv(d[f"l{l}_k_norm"])
        for p in range(npos):
            pos.fill_(p)
            out = ops.attn_decode(ctx, shape, dv(d[f"l{l}_q"][p]), dv(d[f"l{l}_k"][p]), dv(d[f"l{l}_v"][p]), qn, kn,
                                  freq, kc, vc, pos)
            assert _err(out, d[f"l{l}_out"][p]) <= (TOL if kv == "fp16" else 2e-5), (l, p)
            n += 1
    assert n > 0 and ctx.errors() == 0


@pytest.mark.parametrize("name", ["hd64", "hd256"])
def test_deltanet_matches_the_mirror(ops, ctx, name):
    d = load(os.path.join(GOLDEN, f"mirror_layers_{name}.npz"))
    nk, hk, nv, hv, K = (int(d[k]) for k in ("nk", "hk", "nv", "hv", "conv"))
    C = 2 * nk * hk + nv * hv
    dv = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    shape = ops.deltanet_shape(nk, hk, nv, hv, K, float(d["eps"]))
    n = 0
    for l, dn in enumerate(d["layer_types"]):
        if not dn:
            continue
        ring = torch.zeros(K, C, device="cuda")
        S = torch.zeros(nv, hv, hk, device="cuda")
        pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        consts = [dv(d[f"l{l}_{k}"]) for k in ("dt_bias", "ssm_a", "conv_w", "ssm_norm")]
        for p in range(int(d["npos"])):
            pos.fill_(p)
            og = ops.deltanet_step(ctx, shape, dv(d[f"l{l}_qkv"][p]), dv(d[f"l{l}_z"][p]), dv(d[f"l{l}_beta"][p]),
                                   dv(d[f"l{l}_alpha"][p]), *consts, ring, S, pos)
            assert _err(og, d[f"l{l}_out"][p]) <= TOL, (l, p)
            n += 1
    assert n > 0 and ctx.errors() == 0
